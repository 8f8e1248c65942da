"""Math answer-verification environment (reference: ``MathEnvironment``
``nemo_rl/environments/math_environment.py:448`` with the ``HFVerifyWorker`` ``:87``).

Extracts the final answer from the response (last ``\\boxed{...}``, else the
last number) and compares it with the ground truth after normalisation
(whitespace, ``$``, trailing ``.0``, simple fractions evaluated numerically).
Reward 1.0 for a match, 0.0 otherwise.  Responses are decoded with the
tokenizer supplied at construction.
"""

from __future__ import annotations

import re
from fractions import Fraction
from typing import Any, Callable, Optional

import torch

from rl_b200.environments.interfaces import EnvironmentInterface, EnvironmentReturn

__all__ = ["MathEnvironment", "extract_answer", "answers_match"]

_NUM = re.compile(r"-?\d+(?:\.\d+)?(?:/\d+)?")


def _boxed(text: str) -> Optional[str]:
    i = text.rfind("\\boxed{")
    if i < 0:
        return None
    j = i + len("\\boxed{")
    depth = 1
    k = j
    while k < len(text) and depth:
        if text[k] == "{":
            depth += 1
        elif text[k] == "}":
            depth -= 1
        k += 1
    return text[j:k - 1] if depth == 0 else None


def extract_answer(text: str) -> Optional[str]:
    b = _boxed(text)
    if b is not None:
        return b.strip()
    nums = _NUM.findall(text)
    return nums[-1] if nums else None


def _norm(s: str) -> str:
    s = s.strip().replace("$", "").replace(" ", "").replace("\\!", "")
    s = re.sub(r"\\(d|t)?frac\{([^{}]*)\}\{([^{}]*)\}", r"\2/\3", s)
    s = s.rstrip(".")
    return s


def _as_number(s: str) -> Optional[Fraction]:
    try:
        return Fraction(s)
    except (ValueError, ZeroDivisionError):
        return None


def answers_match(pred: Optional[str], truth: Any) -> bool:
    if pred is None or truth is None:
        return False
    a, b = _norm(str(pred)), _norm(str(truth))
    if a == b:
        return True
    na, nb = _as_number(a), _as_number(b)
    return na is not None and nb is not None and na == nb


class MathEnvironment(EnvironmentInterface):
    def __init__(self, cfg: Optional[dict] = None, decode: Optional[Callable[[list[int]], str]] = None):
        self.cfg = cfg or {}
        self.decode = decode

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        rewards, answers = [], []
        for log, meta in zip(message_log_batch, metadata):
            resp = [m for m in log if m["role"] == "assistant"]
            text = "".join(m.get("content") or (self.decode(m["token_ids"].tolist()) if self.decode else "")
                           for m in resp)
            pred = extract_answer(text)
            ok = answers_match(pred, (meta or {}).get("ground_truth"))
            rewards.append(1.0 if ok else 0.0)
            answers.append(pred)
        n = len(message_log_batch)
        return EnvironmentReturn(
            observations=[{"role": "environment", "content": "correct" if r else "incorrect"} for r in rewards],
            metadata=list(metadata), next_stop_strings=[None] * n,
            rewards=torch.tensor(rewards), terminateds=torch.ones(n, dtype=torch.bool), answers=answers)

    def global_post_process_and_metrics(self, batch):
        r = batch["total_reward"]
        return batch, {"accuracy": float(r.mean()) if len(r) else 0.0}
