"""Verifier environments: weighted reward functions (VLM tasks), DAPO math
grading, Jaccard alignment, and a BM25 retrieval tool.

Reference environments (``nemo_rl/environments/``):

* ``vlm_environment.py:117`` ``VLMEnvironment``: ``reward_functions`` is a list
  of ``{name, weight, kwargs}`` over ``format`` / ``exact_alnum`` / ``math_expr``
  / ``bbox_giou`` / ``geo3k``, combined by renormalised weights, graded against
  ``metadata["ground_truth"]`` by a pool of workers;
* ``dapo_math_verifier.py`` (Minerva-normalised ``Answer:`` grading);
* ``code_jaccard_environment.py`` (word-set Jaccard x length ratio);
* ``tools/retriever.py`` ``RAGEnvironment``: ``<retrieve>query</retrieve>``
  answered with the top BM25 documents wrapped in ``<result><1>...</1>...</result>``.

Verification runs on a thread pool of ``num_workers`` (the graders are pure
Python; the pool bounds latency on large batches) in-process.  The graders
terminate the episode after grading; the retriever answers the tool call with
documents and reward 0 and, like the reference, marks the turn terminated.
"""

from __future__ import annotations

import math
import re
from collections import Counter
from concurrent.futures import ThreadPoolExecutor
from functools import partial
from typing import Callable, Optional

import torch

from rl_b200.environments.interfaces import EnvironmentInterface, EnvironmentReturn
from rl_b200.environments.rewards import REWARD_FUNCTIONS, combine_reward_functions, dapo_math_score, jaccard_score

__all__ = ["VLMEnvironment", "DapoMathEnvironment", "CodeJaccardEnvironment", "BM25Retriever", "RAGEnvironment"]


def _assistant_text(log: list[dict], decode) -> str:
    return "".join(str(m.get("content") or (decode(m["token_ids"].tolist()) if decode else ""))
                   for m in log if m["role"] == "assistant")


class _GradingEnvironment(EnvironmentInterface):
    """Single-turn grading of the concatenated assistant text against
    ``metadata["ground_truth"]`` with ``self.grade(response, truth) -> (reward, correct, answer)``."""

    def __init__(self, cfg: Optional[dict] = None, decode: Optional[Callable] = None):
        cfg = dict(cfg or {})
        self.cfg = cfg
        self.decode = decode
        self.pool = ThreadPoolExecutor(max_workers=max(1, int(cfg.get("num_workers", 4))))

    def grade(self, response: str, truth: str) -> tuple[float, bool, Optional[str]]:
        raise NotImplementedError

    def _safe(self, response: str, truth: str):
        try:
            return self.grade(response, truth)
        except Exception:  # noqa: BLE001 - a grader error scores 0, like an unparsable answer
            return 0.0, False, None

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        texts = [_assistant_text(log, self.decode) for log in message_log_batch]
        truths = [str((m or {}).get("ground_truth", "")) for m in metadata]
        out = list(self.pool.map(self._safe, texts, truths))
        n = len(out)
        obs = [{"role": "environment", "content": "Environment: correct" if ok else "Environment: incorrect"}
               for _, ok, _ in out]
        return EnvironmentReturn(obs, list(metadata), [None] * n, torch.tensor([r for r, _, _ in out],
                                                                                dtype=torch.float32),
                                 torch.ones(n, dtype=torch.bool), [a for _, _, a in out])

    def global_post_process_and_metrics(self, batch):
        r = batch["total_reward"].float() if "total_reward" in batch else torch.zeros(0)
        return batch, {"accuracy": float((r > 0.5).float().mean()) if r.numel() else 0.0}

    def shutdown(self) -> None:
        self.pool.shutdown(wait=False)


class VLMEnvironment(_GradingEnvironment):
    """``cfg["reward_functions"]``: ``[{"name": ..., "weight": ..., "kwargs": {...}}]``."""

    def __init__(self, cfg: Optional[dict] = None, decode: Optional[Callable] = None):
        super().__init__(cfg, decode)
        fns = []
        for spec in self.cfg.get("reward_functions") or []:
            name = spec["name"]
            if name not in REWARD_FUNCTIONS:
                raise ValueError(f"invalid reward function {name!r}; known: {sorted(REWARD_FUNCTIONS)}")
            fn = REWARD_FUNCTIONS[name]
            if spec.get("kwargs"):
                fn = partial(fn, **spec["kwargs"])
            fns.append((fn, float(spec.get("weight", 1.0))))
        if not fns:
            raise ValueError("VLMEnvironment needs at least one entry in reward_functions")
        self.verify = combine_reward_functions(fns)

    def grade(self, response, truth):
        r, ok = self.verify(truth, response)
        return r, ok, None


class DapoMathEnvironment(_GradingEnvironment):
    """DAPO math grading (``strict_box_verify`` selects the boxed variant)."""

    def grade(self, response, truth):
        s = dapo_math_score(response, truth, bool(self.cfg.get("strict_box_verify", False)))
        return s["score"], s["acc"], s["pred"]


class CodeJaccardEnvironment(_GradingEnvironment):
    """Alignment of the response with a reference answer (reward in [0, 1];
    "correct" above ``correct_threshold``, default 0.5)."""

    def grade(self, response, truth):
        s = jaccard_score(response, truth)
        return s, s > float(self.cfg.get("correct_threshold", 0.5)), response.strip()


class BM25Retriever:
    """Okapi BM25 over a fixed document list (Robertson & Zaragoza, "The
    Probabilistic Relevance Framework: BM25 and Beyond", 2009):
    score(q, d) = sum over query terms t of idf(t) * tf(t, d) * (k1 + 1) /
    (tf(t, d) + k1 * (1 - b + b * |d| / avgdl)), idf(t) = ln(1 + (N - n_t + 0.5) /
    (n_t + 0.5)).  Terms are lower-cased word characters; scores are a sparse
    product of the document-term weights with the query's idf vector."""

    def __init__(self, documents: list[str], num_result: int = 3, k1: float = 1.5, b: float = 0.75,
                 device: str = "cpu"):
        self.documents = list(documents)
        self.num_result = max(1, min(int(num_result), len(self.documents)))
        self.k1, self.b = float(k1), float(b)
        self.device = device
        self.vocab: dict[str, int] = {}
        rows, cols, tfs = [], [], []
        lengths = []
        for di, doc in enumerate(self.documents):
            c = Counter(self.tokenize(doc))
            lengths.append(sum(c.values()))
            for term, f in c.items():
                ti = self.vocab.setdefault(term, len(self.vocab))
                rows.append(di)
                cols.append(ti)
                tfs.append(float(f))
        N = len(self.documents)
        avgdl = max(1e-9, sum(lengths) / max(1, N))
        df = Counter(cols)
        self.idf = torch.zeros(len(self.vocab))
        for ti, n in df.items():
            self.idf[ti] = math.log(1.0 + (N - n + 0.5) / (n + 0.5))
        dl = torch.tensor([lengths[r] for r in rows], dtype=torch.float32)
        tf = torch.tensor(tfs, dtype=torch.float32)
        w = tf * (self.k1 + 1) / (tf + self.k1 * (1 - self.b + self.b * dl / avgdl))
        self.weights = torch.sparse_coo_tensor(torch.tensor([rows, cols], dtype=torch.long), w,
                                               (N, max(1, len(self.vocab))),
                                               check_invariants=True).coalesce().to(device)

    @staticmethod
    def tokenize(text: str) -> list[str]:
        return re.findall(r"\w+", text.lower())

    def scores(self, query: str) -> torch.Tensor:
        q = torch.zeros(self.weights.shape[1], 1)
        for term in set(self.tokenize(query)):
            ti = self.vocab.get(term)
            if ti is not None:
                q[ti, 0] = self.idf[ti]
        return torch.sparse.mm(self.weights, q.to(self.device)).squeeze(-1).cpu()

    def __call__(self, query: str) -> list[str]:
        top = torch.topk(self.scores(query), self.num_result).indices.tolist()
        return [self.documents[i] for i in top]


class RAGEnvironment(EnvironmentInterface):
    """Retrieval tool: the last assistant message's ``<retrieve>query</retrieve>``
    is answered with the top documents; reward 0 (the task's own environment
    grades the final answer).  Documents: ``cfg["documents"]`` (list of strings)
    or ``cfg["documents_path"]`` (JSONL with ``cfg["text_column"]``, default
    ``text``); BM25 ``k1`` / ``b`` / ``num_results``."""

    def __init__(self, cfg: Optional[dict] = None, decode: Optional[Callable] = None):
        cfg = dict(cfg or {})
        docs = list(cfg.get("documents") or [])
        if cfg.get("documents_path"):
            import json

            col = cfg.get("text_column", "text")
            with open(cfg["documents_path"]) as f:
                docs += [json.loads(line)[col] for line in f if line.strip()]
        if not docs:
            raise ValueError("RAGEnvironment needs documents or documents_path")
        self.decode = decode
        self.retriever = BM25Retriever(docs, int(cfg.get("num_results", 3)), float(cfg.get("k1", 1.5)),
                                       float(cfg.get("b", 0.75)), cfg.get("device", "cpu"))

    @staticmethod
    def format_result(docs: list[str]) -> str:
        body = "".join(f"<{i + 1}>\n{d}\n</{i + 1}>\n" for i, d in enumerate(docs))
        return "<result>\n" + body + "</result>\n"

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        obs = []
        for log in message_log_batch:
            last = log[-1]
            text = str(last.get("content") or (self.decode(last["token_ids"].tolist()) if self.decode else ""))
            m = re.search(r"<retrieve>(.*)</retrieve>", text, re.DOTALL)
            obs.append({"role": "environment",
                        "content": self.format_result(self.retriever(m.group(1))) if m
                        else "No retrieval query found!"})
        n = len(message_log_batch)
        return EnvironmentReturn(obs, list(metadata), [["</retrieve>"]] * n, torch.zeros(n),
                                 torch.ones(n, dtype=torch.bool), [None] * n)


def register(register_environment) -> None:
    register_environment("vlm", lambda c, **k: VLMEnvironment(c, **k))
    register_environment("dapo_math", lambda c, **k: DapoMathEnvironment(c, **k))
    register_environment("code_jaccard", lambda c, **k: CodeJaccardEnvironment(c, **k))
    register_environment("rag", lambda c, **k: RAGEnvironment(c, **k))
    register_environment("retriever", lambda c, **k: RAGEnvironment(c, **k))

