"""Text reward functions for verifier environments.

Each function maps ``(ground_truth, response)`` to ``(reward, is_correct)``
(``is_correct`` None when the function only grades format).  Names and
semantics follow the reference's reward functions
(``nemo_rl/environments/rewards.py``: ``format_reward``,
``exact_answer_alphanumeric_reward``, ``math_expression_reward``,
``bbox_giou_reward``, ``geo3k_reward``, ``combine_reward_functions``) so YAML
configs that name them select the same grading here.  Mathematical equivalence
uses this package's own answer matcher (``math_environment.answers_match``:
exact, normalised-string and rational-number equality) instead of a symbolic
verifier.

Also here:

* ``minerva_normalize`` / ``dapo_math_score``: the answer normalisation of
  Lewkowycz et al., "Solving Quantitative Reasoning Problems with Language
  Models" (2022, appendix: substitutions, removed unit words, ``\\text`` /
  ``\\boxed`` unwrapping) as used by the DAPO math verifier
  (``nemo_rl/environments/dapo_math_verifier.py``), with the ``Answer:`` line
  or, strictly, the last ``\\boxed{}`` of the response's tail;
* ``jaccard_score``: word-set Jaccard similarity times the character-length
  ratio (``nemo_rl/environments/code_jaccard_environment.py``).
"""

from __future__ import annotations

import re
from typing import Callable, Optional

__all__ = ["format_reward", "exact_alnum_reward", "math_expr_reward", "bbox_giou_reward", "geo3k_reward",
           "combine_reward_functions", "REWARD_FUNCTIONS", "last_boxed", "minerva_normalize", "dapo_math_score",
           "jaccard_score"]

RewardFn = Callable[[str, str], "tuple[float, Optional[bool]]"]


def _tagged(response: str, tag: str) -> Optional[str]:
    m = re.search(rf"<{tag}>([\s\S]*)</{tag}>", response)
    return m.group(1) if m else None


def format_reward(ground_truth: str, response: str, think_tag: str = "think",
                  answer_tag: str = "answer") -> tuple[float, Optional[bool]]:
    """0.25 for a ``<think>...</think>`` block plus 0.75 for an ``<answer>...</answer>`` block."""
    r = 0.0
    if _tagged(response, think_tag) is not None:
        r += 0.25
    if _tagged(response, answer_tag) is not None:
        r += 0.75
    return r, None


def exact_alnum_reward(ground_truth: str, response: str, answer_tag: str = "answer") -> tuple[float, bool]:
    """1.0 when the tagged answer equals the ground truth on lower-cased alphanumerics."""
    ans = _tagged(response, answer_tag)
    if ans is None:
        return 0.0, False

    def key(s: str) -> str:
        return "".join(ch for ch in s if ch.isalnum()).lower()

    ok = key(ans) == key(str(ground_truth))
    return (1.0 if ok else 0.0), ok


def math_expr_reward(ground_truth: str, response: str, tag: str = "answer") -> tuple[float, bool]:
    """1.0 when the tagged answer is the same value as the ground truth."""
    from rl_b200.environments.math_environment import answers_match

    ans = _tagged(response, tag)
    if ans is None:
        return 0.0, False
    inner = last_boxed(ans)
    ok = answers_match(inner if inner is not None else ans.strip(), ground_truth)
    return (1.0 if ok else 0.0), ok


def _box(text: str) -> Optional[list[float]]:
    try:
        vals = [float(v) for v in text.replace("[", "").replace("]", "").split(",")]
    except ValueError:
        return None
    return vals if len(vals) == 4 else None


def bbox_giou_reward(ground_truth: str, response: str, giou_penalty_thres: float = 10.0,
                     answer_tag: str = "answer") -> tuple[float, bool]:
    """Generalised IoU of the tagged ``[x1, y1, x2, y2]`` box with the ground
    truth's (plain IoU when the IoU reaches ``giou_penalty_thres``); correct
    above 0.5."""
    ans = _tagged(response, answer_tag)
    g = _box(str(ground_truth))
    p = _box(ans) if ans is not None else None
    if g is None or p is None:
        return 0.0, False
    area = lambda b: (b[2] - b[0]) * (b[3] - b[1])  # noqa: E731
    inter = max(0.0, min(g[2], p[2]) - max(g[0], p[0])) * max(0.0, min(g[3], p[3]) - max(g[1], p[1]))
    union = max(1e-3, area(g) + area(p) - inter)
    iou = inter / union
    score = iou
    if iou < giou_penalty_thres:
        hull = max(1e-3, (max(g[2], p[2]) - min(g[0], p[0])) * (max(g[3], p[3]) - min(g[1], p[1])))
        score = iou - (hull - union) / hull
    return score, score > 0.5


def last_boxed(text: str) -> Optional[str]:
    """Content of the last ``\\boxed{...}`` (braces balanced), or None."""
    i = text.rfind("\\boxed{")
    if i < 0:
        return None
    j = i + len("\\boxed{")
    depth = 1
    for k in range(j, len(text)):
        c = text[k]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return text[j:k]
    return None


def geo3k_reward(ground_truth: str, response: str, format_score: float = 0.1) -> tuple[float, bool]:
    """``(1 - format_score) * accuracy + format_score * format``: format is a
    ``</think>`` followed later by a ``\\boxed{}``; accuracy grades the LAST boxed
    answer."""
    from rl_b200.environments.math_environment import answers_match

    fmt = 1.0 if re.search(r"</think>.*\\boxed\{.*\}", response, re.DOTALL) else 0.0
    ans = last_boxed(response)
    ok = ans is not None and answers_match(ans.strip(), ground_truth)
    return (1.0 - format_score) * (1.0 if ok else 0.0) + format_score * fmt, bool(ok)


def combine_reward_functions(fns: list[tuple[RewardFn, float]]) -> Callable[[str, str], tuple[float, bool]]:
    """Weighted sum (weights renormalised to 1); correct when every function
    that grades correctness says so."""
    if not fns:
        raise ValueError("no reward functions given")
    tot = float(sum(w for _, w in fns))
    if tot <= 0:
        raise ValueError("reward function weights must sum to a positive number")
    ws = [w / tot for _, w in fns]

    def combined(ground_truth: str, response: str) -> tuple[float, bool]:
        out = [fn(ground_truth, response) for fn, _ in fns]
        reward = sum(w * r for w, (r, _) in zip(ws, out))
        return float(reward), all(c for _, c in out if c is not None)

    return combined


REWARD_FUNCTIONS: dict[str, RewardFn] = {
    "format": format_reward,
    "exact_alnum": exact_alnum_reward,
    "math_expr": math_expr_reward,
    "bbox_giou": bbox_giou_reward,
    "geo3k": geo3k_reward,
}


# ---------------------------------------------------------------- Minerva / DAPO
# Substitutions and removed unit words of the Minerva answer normalisation
# (Lewkowycz et al. 2022, appendix); the lists are the method's data.
_MINERVA_SUBS = (("an ", ""), ("a ", ""), (".$", "$"), ("\\$", ""), (r"\ ", ""), (" ", ""), ("mbox", "text"),
                 (",\\text{and}", ","), ("\\text{and}", ","), ("\\text{m}", "\\text{}"))
_MINERVA_REMOVED = ("square", "ways", "integers", "dollars", "mph", "inches", "hours", "km", "units", "\\ldots",
                    "sue", "points", "feet", "minutes", "digits", "cents", "degrees", "cm", "gm", "pounds",
                    "meters", "meals", "edges", "students", "childrentickets", "multiples", "\\text{s}",
                    "\\text{.}", "\\text{\ns}", "\\text{}^2", "\\text{}^3", "\\text{\n}", "\\text{}",
                    r"\mathrm{th}", r"^\circ", r"^{\circ}", r"\;", r",\!", "{,}", '"', "\\dots")


def minerva_normalize(answer: str) -> str:
    """Canonical form of a final answer: the right-hand side of an equation,
    unit words and spacing removed, ``\\text`` / ``\\textbf`` / ``\\overline`` /
    ``\\boxed`` unwrapped, shorthand ``\\frac12`` / ``\\sqrt2`` braced, thousands
    separators dropped from integers."""
    s = answer.split("=")[-1]
    for a, b in _MINERVA_SUBS:
        s = s.replace(a, b)
    for w in _MINERVA_REMOVED:
        s = s.replace(w, "")
    s = re.sub(r"(.*?)(\$)(.*?)(\$)(.*)", "$\\3$", s)
    for cmd in ("text", "textbf", "overline"):
        s = re.sub(r"(\\" + cmd + r"\{)(.*?)(\})", "\\2", s)
    s = re.sub(r"(\\boxed\{)(.*)(\})", "\\2", s)
    s = re.sub(r"(frac)([^{])(.)", "frac{\\2}{\\3}", s)
    s = re.sub(r"(sqrt)([^{])", "sqrt{\\2}", s)
    s = s.replace("$", "")
    if s.replace(",", "").isdigit():
        s = s.replace(",", "")
    return s.strip()


def dapo_math_score(solution: str, ground_truth: str, strict_box: bool = False) -> dict:
    """DAPO-style math grading of the response's last 300 characters: the last
    ``Answer: ...`` line, normalised, against the normalised ground truth (or,
    with ``strict_box``, the last ``\\boxed{}`` of the final 100 characters
    against the raw ground truth).  Returns ``{"score", "acc", "pred"}``."""
    tail = solution[-300:]
    if strict_box:
        pred = last_boxed(tail[-100:])
        ok = pred is not None and pred == ground_truth
    else:
        found = re.findall(r"(?i)Answer\s*:\s*([^\n]+)", tail)
        pred = minerva_normalize(found[-1] if found else "[INVALID]")
        ok = pred == minerva_normalize(str(ground_truth))
    return {"score": 1.0 if ok else 0.0, "acc": bool(ok), "pred": pred}


def jaccard_score(response: str, ground_truth: str) -> float:
    """1.0 on a case-insensitive exact match; otherwise the Jaccard similarity
    of the whitespace-split word sets times min/max of the two lengths."""
    r, g = response.strip().lower(), str(ground_truth).strip().lower()
    if r == g:
        return 1.0
    rw, gw = set(r.split()), set(g.split())
    if not gw:
        return 0.0
    union = len(rw | gw)
    if union == 0:
        return 0.0
    j = len(rw & gw) / union
    ratio = min(len(r), len(g)) / max(len(r), len(g), 1)
    return min(1.0, max(0.0, j * ratio))
