"""Response datasets: raw rows (local files or the Hugging Face cache) formatted
into ``{"messages": [...], "task_name": ...}`` rows for the task processors.

Reference: ``nemo_rl/data/datasets/raw_dataset.py`` (``RawDataset``),
``nemo_rl/data/datasets/response_datasets/__init__.py`` (``DATASET_REGISTRY``,
``load_response_dataset``) and ``nemo_rl/data/datasets/utils.py:97``
(``load_dataset_from_path``).  The registry keys, the constructor keywords of
each dataset (``split``, ``subset``, ``split_validation_size``, ``seed``,
``output_key``, ``variant``, ``repeat``, ...), the ``messages`` row format and the
task names are kept, so the reference's ``data:`` YAML blocks select the same
data here.

Design: rows stay in whatever container they were loaded into (a list of
dicts, or an Arrow-backed ``datasets.Dataset``) and are formatted lazily on
access by ``Rows``, so a million-row corpus is not rewritten in memory before
training starts.  Every named dataset also takes ``data_path``: a local file
(``.jsonl`` / ``.json`` / ``.parquet`` / ``.csv`` / ``.arrow`` / ``.txt``) or a
``save_to_disk`` directory holding the hub dataset's raw columns; without it
the hub id is read through ``datasets.load_dataset``, which in an offline
container resolves only from the local Hugging Face cache.
"""

from __future__ import annotations

import csv
import importlib
import inspect
import json
import os
import random
from typing import Any, Callable, Optional, Sequence

from rl_b200.data.processors import TaskDataSpec, get_processor

__all__ = ["Rows", "load_rows", "RawDataset", "ResponseDataset", "OpenAIFormatDataset", "OpenMathInstruct2Dataset",
           "DAPOMath17KDataset", "DAPOMathAIME2024Dataset", "DeepScalerDataset", "GSM8KDataset", "AIMEDataset",
           "NuminaMath15Dataset", "OpenR1Math220KDataset", "SquadDataset", "Tulu3SftMixtureDataset",
           "HelpSteer3Dataset", "NemoGymDataset", "OasstDataset", "oasst_threads", "ArrowTextDataset",
           "GeneralConversationsJsonlDataset", "NemotronCascade2SFTMathDataset",
           "MegatronSFTPackedDataset", "DATASET_REGISTRY", "load_response_dataset"]


class Rows:
    """Indexable view over ``base`` rows: an optional index list (selection /
    split / repetition) and a chain of per-row formatters applied on access."""

    def __init__(self, base: Any, fmts: Sequence[Callable[[dict], dict]] = (), index: Optional[list[int]] = None):
        self.base = base
        self.fmts = tuple(fmts)
        self.index = index

    def __len__(self) -> int:
        return len(self.index) if self.index is not None else len(self.base)

    def raw(self, i: int) -> dict:
        return self.base[self.index[i] if self.index is not None else i]

    def __getitem__(self, i: int) -> dict:
        if i < 0:
            i += len(self)
        row = self.raw(i)
        for f in self.fmts:
            row = f(row)
        return row

    def __iter__(self):
        for i in range(len(self)):
            yield self[i]

    def map(self, fn: Callable[[dict], dict]) -> "Rows":
        return Rows(self.base, self.fmts + (fn,), self.index)

    def select(self, positions: Sequence[int]) -> "Rows":
        idx = [self.index[p] for p in positions] if self.index is not None else list(positions)
        return Rows(self.base, self.fmts, idx)

    def filter(self, pred: Callable[[dict], bool]) -> "Rows":
        """Keep rows whose formatted value satisfies ``pred`` (one pass)."""
        return self.select([i for i in range(len(self)) if pred(self[i])])

    def repeat(self, n: int) -> "Rows":
        return self.select(list(range(len(self))) * max(1, int(n)))

    def train_test_split(self, test_size: float | int, seed: int) -> tuple["Rows", "Rows"]:
        """Seeded shuffle, then the first ``test_size`` rows (a fraction below 1 or a
        row count) become the test part."""
        n = len(self)
        n_test = int(test_size) if test_size >= 1 else max(1, int(round(n * float(test_size))))
        order = list(range(n))
        random.Random(seed).shuffle(order)
        return self.select(sorted(order[n_test:])), self.select(sorted(order[:n_test]))


def _read_local(path: str) -> list[dict]:
    ext = os.path.splitext(path)[-1].lower()
    if path.lower().endswith(".jsonl.packed") or ext == ".jsonl":
        with open(path, encoding="utf-8") as f:
            return [json.loads(line) for line in f if line.strip()]
    if ext == ".json":
        with open(path, encoding="utf-8") as f:
            txt = f.read()
        try:
            obj = json.loads(txt)
        except json.JSONDecodeError:  # JSON lines under a .json name
            return [json.loads(line) for line in txt.splitlines() if line.strip()]
        if isinstance(obj, dict):  # columnar {"col": [...]}
            cols = list(obj)
            return [dict(zip(cols, vals)) for vals in zip(*(obj[c] for c in cols))]
        return list(obj)
    if ext == ".parquet":
        import pyarrow.parquet as pq

        return pq.read_table(path).to_pylist()
    if ext == ".arrow":
        import pyarrow as pa

        with pa.memory_map(path) as src:
            try:
                return pa.ipc.open_stream(src).read_all().to_pylist()
            except pa.ArrowInvalid:
                return pa.ipc.open_file(src).read_all().to_pylist()
    if ext == ".csv":
        with open(path, encoding="utf-8", newline="") as f:
            return list(csv.DictReader(f))
    if ext == ".txt":
        with open(path, encoding="utf-8") as f:
            return [{"text": line.rstrip("\n")} for line in f]
    raise ValueError(f"unsupported data file type {ext!r} ({path})")


def load_rows(data_path: str, subset: Optional[str] = None, split: Optional[str] = "train") -> Rows:
    """Rows of a local file, a ``save_to_disk`` directory, or a Hugging Face
    dataset id (resolved through the local cache when offline)."""
    if os.path.isfile(data_path):
        if subset is not None:
            raise ValueError("a subset applies only to Hugging Face datasets")
        return Rows(_read_local(data_path))
    import datasets

    if os.path.isdir(data_path) and (os.path.exists(os.path.join(data_path, "dataset_info.json"))
                                      or os.path.exists(os.path.join(data_path, "dataset_dict.json"))):
        ds = datasets.load_from_disk(data_path)
    else:
        try:
            ds = datasets.load_dataset(data_path, subset) if subset else datasets.load_dataset(data_path)
        except Exception as e:  # noqa: BLE001 - say what to do offline
            raise RuntimeError(
                f"could not load dataset {data_path!r} ({type(e).__name__}: {e}); without network access pass "
                f"data_path pointing at a local copy of its rows (jsonl / json / parquet / csv / arrow) or a "
                f"save_to_disk directory") from e
    if isinstance(ds, datasets.DatasetDict):
        if split:
            ds = ds[split]
        elif "train" in ds:
            ds = ds["train"]
    return Rows(ds)


def _messages(user: str, assistant: Any, system: Optional[str] = None) -> list[dict]:
    msgs = [{"role": "system", "content": system}] if system is not None else []
    return msgs + [{"role": "user", "content": user}, {"role": "assistant", "content": assistant}]


class RawDataset:
    """A loaded dataset: formatted ``dataset`` rows, an optional ``val_dataset``
    split off it, and (after ``set_task_spec`` / ``set_processor``) the task's
    prompt spec and processor."""

    task_name: str = "default"
    dataset: Rows
    val_dataset: Optional[Rows] = None
    preprocessor: Optional[Callable[[dict], dict]] = None

    def split_train_validation(self, test_size: float | int, seed: int) -> None:
        if test_size and test_size > 0:
            self.dataset, self.val_dataset = self.dataset.train_test_split(test_size, seed)

    def set_task_spec(self, data_config: dict) -> None:
        self.data_config = data_config
        self.task_spec = TaskDataSpec(task_name=self.task_name, prompt_file=data_config.get("prompt_file"),
                                      system_prompt_file=data_config.get("system_prompt_file"))

    def set_processor(self) -> None:
        self.processor = get_processor((getattr(self, "data_config", None) or {}).get("processor", "default"))


class _HubResponseDataset(RawDataset):
    """A hub dataset read from ``data_path`` or its hub id, formatted row by row."""

    HUB: str = ""
    SUBSET: Optional[str] = None
    SPLIT: str = "train"

    def _load(self, data_path: Optional[str], subset: Optional[str], split: Optional[str]) -> Rows:
        if data_path:
            return load_rows(data_path, None if os.path.isfile(data_path) else subset,
                             None if os.path.isfile(data_path) else split)
        return load_rows(self.HUB, subset, split)

    def format_data(self, row: dict) -> dict:  # pragma: no cover - overridden
        raise NotImplementedError


class OpenMathInstruct2Dataset(_HubResponseDataset):
    HUB = "nvidia/OpenMathInstruct-2"

    def __init__(self, output_key: str = "expected_answer", split: str = "train_1M",
                 split_validation_size: float = 0.05, seed: int = 42, data_path: Optional[str] = None, **_):
        if split not in ("train", "train_1M", "train_2M", "train_5M"):
            raise ValueError(f"OpenMathInstruct-2 split must be train / train_1M / train_2M / train_5M, not {split!r}")
        self.task_name = "OpenMathInstruct-2"
        self.output_key = output_key
        self.dataset = self._load(data_path, None, split).map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        return {"messages": _messages(row["problem"], row[self.output_key]), "task_name": self.task_name}


class DAPOMath17KDataset(_HubResponseDataset):
    HUB = "BytedTsinghua-SIA/DAPO-Math-17k"
    TASK = "DAPOMath17K"

    def __init__(self, data_path: Optional[str] = None, **_):
        self.task_name = self.TASK
        self.dataset = self._load(data_path, None, "train").map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        # verl-style rows: prompt = [{"role": "user", "content": ...}], reward_model.ground_truth
        return {"messages": _messages(row["prompt"][0]["content"], row["reward_model"]["ground_truth"]),
                "task_name": self.task_name}


class DAPOMathAIME2024Dataset(DAPOMath17KDataset):
    HUB = "BytedTsinghua-SIA/AIME-2024"
    TASK = "DAPOMathAIME2024"


class DeepScalerDataset(_HubResponseDataset):
    HUB = "agentica-org/DeepScaleR-Preview-Dataset"

    def __init__(self, data_path: Optional[str] = None, **_):
        self.task_name = "DeepScaler"
        self.dataset = self._load(data_path, None, "train").map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        return {"messages": _messages(row["problem"], row["answer"]), "task_name": self.task_name}


def _after_hashes(text: str) -> Optional[str]:
    """GSM8K answers end in ``#### <final answer>``."""
    return text.split("####", 1)[1].strip() if "####" in text else None


class GSM8KDataset(_HubResponseDataset):
    HUB = "openai/gsm8k"

    def __init__(self, subset: Optional[str] = "main", split: str = "train", extract_answer: bool = True,
                 data_path: Optional[str] = None, **_):
        self.task_name = "gsm8k"
        self.extract_answer = extract_answer
        self.dataset = self._load(data_path, subset or "main", split).map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        ans = _after_hashes(row["answer"]) if self.extract_answer else row["answer"]
        return {"messages": _messages(row["question"], ans), "task_name": self.task_name}


class AIMEDataset(_HubResponseDataset):
    _VARIANTS = {"2024": ("HuggingFaceH4/aime_2024", None, "train", "problem"),
                 "2025": ("opencompass/AIME2025", ("AIME2025-I", "AIME2025-II"), "test", "question"),
                 "2026": ("MathArena/aime_2026", None, "train", "problem")}

    def __init__(self, variant: str = "2024", repeat: int = 1, data_path: Optional[str] = None, **_):
        if variant not in self._VARIANTS:
            raise ValueError(f"AIME variant must be one of {sorted(self._VARIANTS)}, not {variant!r}")
        repo, subsets, split, self.input_key = self._VARIANTS[variant]
        self.task_name = f"AIME{variant}"
        if data_path:
            rows = self._load(data_path, None, split)
        elif subsets:
            parts = [load_rows(repo, s, split) for s in subsets]
            rows = Rows([r for p in parts for r in p])
        else:
            rows = load_rows(repo, None, split)
        self.dataset = rows.map(self.format_data).repeat(repeat)
        self.val_dataset = None

    def format_data(self, row):
        key = self.input_key if self.input_key in row else ("problem" if "problem" in row else "question")
        return {"messages": _messages(row[key], str(row["answer"])), "task_name": self.task_name}


class NuminaMath15Dataset(_HubResponseDataset):
    HUB = "AI-MO/NuminaMath-1.5"
    UNVERIFIABLE = frozenset({"proof", "notfound"})

    def __init__(self, split: str = "train", verifiable_only: bool = True, require_valid: bool = True,
                 split_validation_size: float = 0.0, seed: int = 42, data_path: Optional[str] = None, **_):
        self.task_name = "NuminaMath-1.5"
        rows = self._load(data_path, None, split)
        if verifiable_only:
            rows = rows.filter(self._verifiable)
        if require_valid:
            rows = rows.filter(lambda r: r.get("problem_is_valid") == "Yes" and r.get("solution_is_valid") == "Yes")
        self.dataset = rows.map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    @classmethod
    def _verifiable(cls, row) -> bool:
        ans = (row.get("answer") or "").strip()
        if not ans or ans.lower() in cls.UNVERIFIABLE:
            return False
        return (row.get("question_type") or "").strip().lower() != "proof"

    def format_data(self, row):
        return {"messages": _messages(row["problem"], row["answer"]), "task_name": self.task_name}


class OpenR1Math220KDataset(_HubResponseDataset):
    HUB = "open-r1/OpenR1-Math-220k"

    def __init__(self, subset: Optional[str] = "default", split: str = "train", split_validation_size: float = 0.0,
                 seed: int = 42, data_path: Optional[str] = None, **_):
        self.task_name = "OpenR1-Math-220k"
        self.dataset = self._load(data_path, subset or "default", split).map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        return {"messages": _messages(row["problem"], row["answer"]), "task_name": self.task_name}


class SquadDataset(_HubResponseDataset):
    HUB = "rajpurkar/squad"

    def __init__(self, split: str = "train", data_path: Optional[str] = None, **_):
        self.task_name = "squad"
        self.dataset = self._load(data_path, None, split).map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        return {"messages": _messages(row["question"], row["answers"]["text"][0], system=row["context"]),
                "task_name": self.task_name}


class Tulu3SftMixtureDataset(_HubResponseDataset):
    HUB = "allenai/tulu-3-sft-mixture"

    def __init__(self, split_validation_size: float = 0.05, seed: int = 42, max_samples: Optional[int] = None,
                 data_path: Optional[str] = None, **_):
        self.task_name = "tulu3_sft_mixture"
        rows = self._load(data_path, None, "train")
        if max_samples:
            order = list(range(len(rows)))
            random.Random(seed).shuffle(order)
            rows = rows.select(order[:min(int(max_samples), len(rows))])
        self.dataset = rows.map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        msgs = row["messages"]
        if not msgs or msgs[-1]["role"] != "assistant":
            raise ValueError("tulu-3 rows must end with an assistant turn")
        return {"messages": msgs, "task_name": self.task_name}


class HelpSteer3Dataset(_HubResponseDataset):
    """HelpSteer3 preference rows as RL prompts: the context, with the preferred
    response (``overall_preference`` < 0: response1; > 0: response2; 0: response1)
    kept as the reference answer."""

    HUB = "nvidia/HelpSteer3"

    def __init__(self, split: str = "train", data_path: Optional[str] = None, **_):
        self.task_name = "HelpSteer3"
        self.dataset = self._load(data_path, "preference", split).map(self.format_data)
        self.val_dataset = None

    def format_data(self, row):
        pref = row["overall_preference"]
        chosen = row["response2"] if pref > 0 else row["response1"]
        ctx = row["context"]
        ctx = [{"role": "user", "content": ctx}] if isinstance(ctx, str) else ctx
        return {"context": ctx, "response": [{"role": "assistant", "content": chosen}], "task_name": self.task_name}


def _task_name_of_path(path: str) -> str:
    name = "-".join(path.rstrip("/").split("/")[-2:]).split(".")[0]
    return name.lstrip("-") or "dataset"


class ResponseDataset(RawDataset):
    """Generic ``{input_key: prompt, output_key: answer}`` rows (or rows that
    already carry ``messages``) from a local file or a hub id."""

    def __init__(self, data_path: str, input_key: str = "input", output_key: str = "output",
                 subset: Optional[str] = None, split: Optional[str] = None, split_validation_size: float = 0,
                 seed: int = 42, **_):
        self.input_key, self.output_key = input_key, output_key
        self.task_name = _task_name_of_path(data_path)
        self.dataset = load_rows(data_path, subset, split).map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        if "messages" in row:
            return {**row, "task_name": row.get("task_name") or self.task_name}
        return {"messages": _messages(row[self.input_key], row[self.output_key]), "task_name": self.task_name}


class OpenAIFormatDataset(RawDataset):
    """Chat rows ``{chat_key: [{"role", "content"[, "tool_calls"]}...]}``, each row kept
    exactly as written (no schema filling), with an optional system prompt."""

    def __init__(self, data_path: str, chat_key: str = "messages", system_key: Optional[str] = None,
                 system_prompt: Optional[str] = None, tool_key: str = "tools", split_validation_size: float = 0,
                 seed: int = 42, **_):
        self.chat_key, self.system_key, self.system_prompt, self.tool_key = chat_key, system_key, system_prompt, tool_key
        self.task_name = _task_name_of_path(data_path)
        self.dataset = load_rows(data_path, None, None).map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        msgs = list(row[self.chat_key])
        sys_txt = row.get(self.system_key) if self.system_key else None
        sys_txt = sys_txt or self.system_prompt
        if sys_txt and (not msgs or msgs[0]["role"] != "system"):
            msgs = [{"role": "system", "content": sys_txt}] + msgs
        out = {"messages": msgs, "task_name": self.task_name}
        if row.get(self.tool_key):
            out["tools"] = row[self.tool_key]
        return out


def _rows_of_files(pattern: str) -> list[dict]:
    """Rows of every local file a path or glob names, in sorted path order."""
    import glob

    paths = sorted(glob.glob(pattern)) if any(c in pattern for c in "*?[") else [pattern]
    if not paths:
        raise FileNotFoundError(f"no data files match {pattern!r}")
    rows: list[dict] = []
    for p in paths:
        rows.extend(_read_local(p))
    return rows


class NemoGymDataset(RawDataset):
    """NeMo-Gym task rows: each row's ``extra_env_info`` payload (a JSON string, or
    already a dict) is handed to the Gym environment unparsed here; the processor
    (``nemo_gym_data_processor``) parses it.

    Reference: ``nemo_rl/data/datasets/response_datasets/nemogym_dataset.py:22``
    (task name from the last two path components, ``.jsonl`` rows kept as raw
    strings, an ``extra_env_info`` or ``text`` column otherwise, ``repeat``)."""

    def __init__(self, data_path: str, repeat: int = 1, **_):
        self.task_name = _task_name_of_path(data_path)
        if os.path.isfile(data_path) and data_path.lower().endswith(".jsonl"):
            with open(data_path, encoding="utf-8") as f:  # raw lines: the payload is parsed later
                base = [{"extra_env_info": line.rstrip("\n")} for line in f if line.strip()]
        else:
            rows = load_rows(data_path, None, None)
            first = rows[0] if len(rows) else {}
            col = "extra_env_info" if "extra_env_info" in first else "text" if "text" in first else None
            if col is None:
                raise ValueError(f"a NeMo-Gym dataset needs an 'extra_env_info' or 'text' column; {data_path!r} "
                                 f"has {sorted(first)}")
            base = [{"extra_env_info": rows.raw(i)[col]} for i in range(len(rows))]
        task = self.task_name
        self.dataset = Rows(base).map(lambda r: {"extra_env_info": r["extra_env_info"], "task_name": task})
        if int(repeat) > 1:
            self.dataset = self.dataset.repeat(int(repeat))
        self.val_dataset = None


OASST_SYSTEM_PROMPT = ("A chat between a curious user and an artificial intelligence assistant. The assistant gives "
                       "helpful, detailed, and polite answers to the user's questions.\n\n")
_OASST_ROLES = {"prompter": "user", "assistant": "assistant"}


def oasst_threads(tree: dict) -> list[list[dict]]:
    """Every root-to-leaf thread of one OpenAssistant message tree as a message
    list (system prompt first), depth first with replies in file order.

    The tree is ``{"prompt": node}`` or a bare node ``{"text", "role", "replies"}``;
    ``prompter`` turns become ``user``.  Written with an explicit stack, so deep
    trees need no recursion."""
    root = tree.get("prompt", tree if ("text" in tree and "role" in tree) else None)
    if root is None:
        return [[{"role": "system", "content": OASST_SYSTEM_PROMPT}]]
    out: list[list[dict]] = []
    stack = [(root, [{"role": "system", "content": OASST_SYSTEM_PROMPT}])]
    while stack:
        node, path = stack.pop()
        if node["role"] not in _OASST_ROLES:
            raise ValueError(f"unknown OASST role {node['role']!r}")
        path = path + [{"role": _OASST_ROLES[node["role"]], "content": node["text"]}]
        replies = [r for r in node.get("replies", []) if "text" in r and "role" in r]
        if not replies:
            out.append(path)
        for child in reversed(replies):  # reversed onto the stack = file order off it
            stack.append((child, path))
    return out


class OasstDataset(RawDataset):
    """OpenAssistant conversation trees flattened into one row per thread (threads
    with a single turn after the system prompt are dropped).

    Reference: ``nemo_rl/data/datasets/response_datasets/oasst.py:96`` (the
    ``2023-04-12_oasst_all.trees.jsonl.gz`` file of ``OpenAssistant/oasst1``,
    ``split_validation_size``, ``seed``).  ``data_path`` names a local copy of the
    trees file (``.jsonl`` or ``.jsonl.gz``); without it the file is looked up in
    the local Hugging Face hub cache."""

    HUB_FILE = "2023-04-12_oasst_all.trees.jsonl.gz"

    def __init__(self, split_validation_size: float = 0.05, seed: int = 42, data_path: Optional[str] = None, **_):
        self.task_name = "oasst"
        path = data_path or self._cached_file()
        opener = __import__("gzip").open if path.endswith(".gz") else open
        rows = []
        with opener(path, "rt", encoding="utf-8") as f:
            for line in f:
                if line.strip():
                    for thread in oasst_threads(json.loads(line)):
                        if len(thread) > 2:
                            rows.append({"messages": thread, "task_name": self.task_name})
        self.dataset = Rows(rows)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def _cached_file(self) -> str:
        try:
            from huggingface_hub import hf_hub_download

            return hf_hub_download("OpenAssistant/oasst1", self.HUB_FILE, repo_type="dataset", local_files_only=True)
        except Exception as e:  # noqa: BLE001 - say what to do offline
            raise RuntimeError(f"OASST trees file not in the local hub cache ({type(e).__name__}); pass data_path "
                               f"pointing at a copy of {self.HUB_FILE}") from e


class ArrowTextDataset(RawDataset):
    """Raw text rows (``text_key``) as single assistant turns for distillation / SFT,
    optionally packed: consecutive non-empty rows joined with newlines until the
    pack reaches ``characters_per_sample`` characters.

    Reference: ``nemo_rl/data/datasets/response_datasets/arrow_text_dataset.py:33``
    (``data_files`` path / glob / hub id, ``subset``, ``split``, ``text_key``,
    ``characters_per_sample``, task ``x_token``)."""

    def __init__(self, data_files: str, subset: Optional[str] = None, split: str = "train", text_key: str = "text",
                 characters_per_sample: Optional[int] = None, split_validation_size: float = 0.0, seed: int = 42,
                 **_):
        self.task_name, self.text_key = "x_token", text_key
        if os.path.isfile(data_files) or any(c in data_files for c in "*?["):
            raw = Rows(_rows_of_files(data_files))
        else:
            raw = load_rows(data_files, subset, split)
        texts = [t for t in (raw.raw(i).get(text_key) for i in range(len(raw))) if isinstance(t, str) and t]
        if characters_per_sample and int(characters_per_sample) > 0:
            packs, buf, n = [], [], 0
            for t in texts:
                buf.append(t)
                n += len(t)
                if n >= int(characters_per_sample):
                    packs.append("\n".join(buf))
                    buf, n = [], 0
            if buf:
                packs.append("\n".join(buf))
            texts = packs
        task = self.task_name
        self.dataset = Rows([{"text": t} for t in texts]).map(
            lambda r: {"messages": [{"role": "assistant", "content": r["text"]}], "task_name": task})
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)


# canonical media tags, the aliases rows may use for them, and the role names
# ShareGPT-style rows use
MEDIA_TAGS = ("image", "video", "audio", "video-audio")
MEDIA_TAG_ALIASES = {"speech": "audio", "speeches": "audio", "sound": "audio", "audios": "audio",
                     "images": "image", "videos": "video"}
CONVERSATION_ROLES = {"user": "user", "assistant": "assistant", "human": "user", "gpt": "assistant",
                      "agent": "assistant"}


class GeneralConversationsJsonlDataset(RawDataset):
    """ShareGPT-style JSONL rows ``{"conversations": [{"from", "value"}...], <media
    key>: file or [files]}`` turned into OpenAI-style messages whose content is a
    list of ``{"type": "text", "text": ...}`` / ``{"type": m, m: path}`` fragments,
    the ``<image>`` / ``<video>`` / ``<audio>`` / ``<video-audio>`` tags in a turn
    consumed in order from the row's media lists (aliases such as ``sound`` or
    ``images`` map to the canonical tag; ``video-audio`` yields a video and an
    audio fragment).  Media names that are not files are looked up under
    ``media_data_dir``.

    Reference: ``nemo_rl/data/datasets/response_datasets/
    general_conversations_dataset.py:147`` (``_datum_preprocessor`` ``:231``)."""

    task_name = "general-conversation-jsonl"

    def __init__(self, data_path: str, media_data_dir: Optional[str] = None, split_validation_size: float = 0,
                 seed: int = 42, **_):
        import re

        self.media_data_dir = media_data_dir
        self._split = re.compile("(" + "|".join(re.escape(f"<{t}>") for t in MEDIA_TAGS) + ")")
        self.dataset = load_rows(data_path, None, None).map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def _media(self, tag: str, name: Any) -> list[dict]:
        if (self.media_data_dir is not None and isinstance(name, str) and not os.path.isfile(name)
                and os.path.isfile(os.path.join(self.media_data_dir, name))):
            name = os.path.join(self.media_data_dir, name)
        return [{"type": t, t: name} for t in tag.split("-")]

    def format_data(self, row: dict) -> dict:
        media: dict[str, list] = {}
        for key, val in row.items():
            tag = MEDIA_TAG_ALIASES.get(key, key)
            if tag in MEDIA_TAGS and val is not None and not (key != tag and tag in row):
                media[tag] = list(val) if isinstance(val, (list, tuple)) else [val]
        used = {t: 0 for t in media}
        msgs = []
        for turn in row.get("conversations", []):
            role = CONVERSATION_ROLES.get(turn["from"])
            if role is None:
                raise ValueError(f"unknown conversation role {turn['from']!r}")
            text = turn["value"]
            for alias, tag in MEDIA_TAG_ALIASES.items():
                text = text.replace(f"<{alias}>", f"<{tag}>")
            content = []
            for part in self._split.split(text):
                tag = part[1:-1] if part.startswith("<") and part[1:-1] in MEDIA_TAGS else None
                if tag is not None:
                    if tag not in media or used[tag] >= len(media[tag]):
                        raise ValueError(f"{part} in a turn but the row has no {tag!r} entry left for it")
                    content += self._media(tag, media[tag][used[tag]])
                    used[tag] += 1
                elif part.strip():
                    content.append({"type": "text", "text": part})
            msgs.append({"role": role, "content": content})
        return {"messages": msgs, "task_name": self.task_name}


class NemotronCascade2SFTMathDataset(_HubResponseDataset):
    """``nvidia/Nemotron-Cascade-2-SFT-Data`` (``math`` subset): chat rows already in
    OpenAI message form ending with the assistant turn; ``max_samples`` draws a
    seeded random subset before the validation split.

    Reference: ``nemo_rl/data/datasets/response_datasets/nemotron_cascade2_sft.py``."""

    HUB, SUBSET = "nvidia/Nemotron-Cascade-2-SFT-Data", "math"

    def __init__(self, split: str = "train", split_validation_size: float = 0.05, seed: int = 42,
                 max_samples: Optional[int] = None, data_path: Optional[str] = None, **_):
        self.task_name = "Nemotron-Cascade-2-SFT-Math"
        rows = self._load(data_path, self.SUBSET, split)
        if max_samples is not None and int(max_samples) > 0:
            order = list(range(len(rows)))
            random.Random(seed).shuffle(order)
            rows = rows.select(order[:min(int(max_samples), len(rows))])
        self.dataset = rows.map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        msgs = row["messages"]
        if not msgs or msgs[-1]["role"] != "assistant":
            raise ValueError(f"expected the last message to be the assistant's, got {msgs}")
        return {"messages": msgs, "task_name": self.task_name}


class MegatronSFTPackedDataset(RawDataset):
    """Megatron-LM offline-packed SFT records (``chat_key`` holds one packed message
    list, system message first, assistant message last, string contents), turned
    into pre-shifted rows by ``megatron_sft_packed_preprocessor`` with the
    ``data_config["megatron_sft"]`` prompt format.

    Reference: ``nemo_rl/data/datasets/response_datasets/megatron_sft_packed.py:29``."""

    def __init__(self, data_path: str, chat_key: str, subset: Optional[str] = None, split: Optional[str] = None,
                 split_validation_size: float = 0, seed: int = 42, context_parallel_size: Optional[int] = None,
                 **_):
        if context_parallel_size is None or int(context_parallel_size) < 1:
            raise ValueError("packed Megatron SFT data needs the policy's context_parallel_size (>= 1)")
        self.context_parallel_size, self.chat_key = int(context_parallel_size), chat_key
        self.task_name = "megatron_sft_packed"
        self.dataset = load_rows(data_path, subset, split).map(self.format_data)
        self.val_dataset = None
        self.split_train_validation(split_validation_size, seed)

    def format_data(self, row):
        msgs = list(row[self.chat_key])
        if not msgs or msgs[0]["role"] != "system":
            raise ValueError("packed Megatron SFT records must start with a system message")
        if msgs[-1]["role"] != "assistant":
            raise ValueError("packed Megatron SFT records must end with an assistant message")
        if any(not isinstance(m["content"], str) for m in msgs):
            raise ValueError("packed Megatron SFT records need string contents")
        return {"packed_messages": msgs, "task_name": self.task_name}

    def set_processor(self) -> None:
        import functools

        from rl_b200.data.megatron_sft_packed import megatron_sft_packed_preprocessor, resolve_prompt_format

        cfg = dict((getattr(self, "data_config", None) or {}).get("megatron_sft") or {})
        unknown = set(cfg) - {"prompt_format", "override_pad_token"}
        if unknown:
            raise ValueError(f"unknown megatron_sft settings: {sorted(unknown)}")
        if "prompt_format" not in cfg:
            raise ValueError("data.megatron_sft.prompt_format is required for megatron_sft_packed")
        resolve_prompt_format(cfg["prompt_format"], cfg.get("override_pad_token"))
        self.processor = functools.partial(megatron_sft_packed_preprocessor, prompt_format=cfg["prompt_format"],
                                           pad_token=cfg.get("override_pad_token"),
                                           context_parallel_size=self.context_parallel_size)


DATASET_REGISTRY: dict[str, Callable[..., RawDataset]] = {
    "OpenMathInstruct-2": OpenMathInstruct2Dataset,
    "DAPOMath17K": DAPOMath17KDataset,
    "DAPOMathAIME2024": DAPOMathAIME2024Dataset,
    "DeepScaler": DeepScalerDataset,
    "GSM8K": GSM8KDataset,
    "gsm8k": GSM8KDataset,
    "AIME2024": lambda **kw: AIMEDataset(variant="2024", **{k: v for k, v in kw.items() if k != "variant"}),
    "AIME2025": lambda **kw: AIMEDataset(variant="2025", **{k: v for k, v in kw.items() if k != "variant"}),
    "AIME2026": lambda **kw: AIMEDataset(variant="2026", **{k: v for k, v in kw.items() if k != "variant"}),
    "NuminaMath-1.5": NuminaMath15Dataset,
    "OpenR1-Math-220k": OpenR1Math220KDataset,
    "squad": SquadDataset,
    "tulu3_sft_mixture": Tulu3SftMixtureDataset,
    "HelpSteer3": HelpSteer3Dataset,
    "openai_format": OpenAIFormatDataset,
    "ResponseDataset": ResponseDataset,
    "NemoGymDataset": NemoGymDataset,
    "open_assistant": OasstDataset,
    "arrow_text": ArrowTextDataset,
    "general-conversation-jsonl": GeneralConversationsJsonlDataset,
    "Nemotron-Cascade-2-SFT-Math": NemotronCascade2SFTMathDataset,
    "megatron_sft_packed": MegatronSFTPackedDataset,
}


def _external_class(dotted: str) -> Callable[..., RawDataset]:
    mod, _, name = dotted.rpartition(".")
    try:
        cls = getattr(importlib.import_module(mod), name)
    except (ImportError, AttributeError) as e:
        raise ValueError(f"cannot import dataset class {dotted!r}: {e}") from e
    if not inspect.isclass(cls):
        raise ValueError(f"{dotted!r} is not a class")
    return cls


def load_response_dataset(data_config: dict, *, context_parallel_size: Optional[int] = None) -> RawDataset:
    """Build the dataset a ``data.train`` / ``data.validation`` entry names:
    a registry key, or a dotted import path of a ``RawDataset`` subclass; then bind
    its task spec (prompt / system prompt files) and processor.
    ``context_parallel_size`` (the policy's) is passed to ``megatron_sft_packed``."""
    name = data_config["dataset_name"]
    if name in DATASET_REGISTRY:
        factory = DATASET_REGISTRY[name]
    elif "." in name:
        factory = _external_class(name)
    else:
        raise ValueError(f"unknown dataset_name {name!r}: use one of {sorted(DATASET_REGISTRY)}, 'ResponseDataset' "
                         f"for a local file, or a dotted path to a dataset class")
    kwargs = {k: v for k, v in data_config.items() if k not in ("dataset_name", "megatron_sft")}
    if name == "megatron_sft_packed":
        kwargs["context_parallel_size"] = context_parallel_size
    ds = factory(**kwargs)
    ds.set_task_spec(data_config)
    ds.set_processor()
    return ds
