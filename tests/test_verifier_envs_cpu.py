"""Verifier environments and reward functions: the documented behaviours of the
reference's VLM reward functions, DAPO (Minerva-normalised) math grading, Jaccard
alignment and the BM25 retrieval tool (CPU)."""

from __future__ import annotations

import json

import pytest
import torch

from rl_b200.environments.registry import make_environment
from rl_b200.environments.rewards import (bbox_giou_reward, combine_reward_functions, dapo_math_score,
                                          exact_alnum_reward, format_reward, geo3k_reward, jaccard_score,
                                          last_boxed, math_expr_reward, minerva_normalize)


def _log(text):
    return [{"role": "user", "content": "q"}, {"role": "assistant", "content": text}]


def test_reward_functions():
    assert format_reward("x", "<think>a</think><answer>b</answer>") == (1.0, None)
    assert format_reward("x", "<answer>b</answer>") == (0.75, None)
    assert exact_alnum_reward("Blue Car", "<answer> blue-car! </answer>") == (1.0, True)
    assert exact_alnum_reward("3", "no tags") == (0.0, False)
    assert math_expr_reward("1/2", "<answer>0.5</answer>") == (1.0, True)
    assert math_expr_reward("3", "<answer>\\boxed{3}</answer>") == (1.0, True)
    r, ok = bbox_giou_reward("[0,0,1,1]", "<answer>[0,0,1,1]</answer>")
    assert r == pytest.approx(1.0) and ok
    r, ok = bbox_giou_reward("[0,0,1,1]", "<answer>[2,2,3,3]</answer>")
    assert r < 0 and not ok  # disjoint: GIoU penalises the empty hull area
    r, ok = geo3k_reward("7", "<think>..</think> so \\boxed{5} no, \\boxed{7}")
    assert r == pytest.approx(1.0) and ok
    r, ok = geo3k_reward("7", "\\boxed{7}")  # right answer, no </think>: 0.9
    assert r == pytest.approx(0.9) and ok
    assert last_boxed("a \\boxed{\\frac{1}{2}} b") == "\\frac{1}{2}"
    comb = combine_reward_functions([(format_reward, 1.0), (exact_alnum_reward, 3.0)])
    r, ok = comb("cat", "<answer>cat</answer>")
    assert r == pytest.approx(0.25 * 0.75 + 0.75 * 1.0) and ok


def test_minerva_normalisation_and_dapo_score():
    assert minerva_normalize("x = 10 \\text{ dollars}") == "10"
    assert minerva_normalize("\\boxed{1,000}") == "1000"
    assert minerva_normalize("\\frac12") == "\\frac{1}{2}"
    assert dapo_math_score("... so Answer: 1,000 dollars", "1000")["acc"]
    assert not dapo_math_score("Answer: 12", "13")["acc"]
    assert dapo_math_score("no answer line", "13")["pred"] == "[INVALID]"
    assert dapo_math_score("thus \\boxed{42}", "42", strict_box=True)["score"] == 1.0


def test_jaccard_score():
    assert jaccard_score("Return X", "return x") == 1.0
    assert jaccard_score("a b c", "") == 0.0
    s = jaccard_score("def f(x): return x", "def f(x): return x + 1")
    assert 0.0 < s < 1.0


def test_vlm_environment_weighted_functions():
    env = make_environment("vlm", {"num_workers": 2, "reward_functions": [
        {"name": "format", "weight": 1.0}, {"name": "exact_alnum", "weight": 1.0}]})
    out = env.step([_log("<think>t</think><answer>dog</answer>"), _log("<answer>cat</answer>")],
                   [{"ground_truth": "dog"}, {"ground_truth": "dog"}])
    assert torch.allclose(out.rewards, torch.tensor([1.0, 0.375]))
    assert out.observations[0]["content"] == "Environment: correct" and bool(out.terminateds.all())
    with pytest.raises(ValueError):
        make_environment("vlm", {"reward_functions": [{"name": "nope", "weight": 1}]})


def test_dapo_and_jaccard_environments():
    env = make_environment("dapo_math", {})
    out = env.step([_log("Answer: 7"), _log("Answer: 8")], [{"ground_truth": "7"}, {"ground_truth": "7"}])
    assert out.rewards.tolist() == [1.0, 0.0] and out.answers == ["7", "8"]
    env = make_environment("code_jaccard", {})
    out = env.step([_log("print(1)")], [{"ground_truth": "print(1)"}])
    assert out.rewards.tolist() == [1.0]


def test_bm25_retrieval_tool(tmp_path):
    docs = ["the capital of france is paris", "bananas are yellow fruit", "paris is in europe and france"]
    p = tmp_path / "docs.jsonl"
    p.write_text("\n".join(json.dumps({"text": d}) for d in docs))
    env = make_environment("rag", {"documents_path": str(p), "num_results": 2})
    out = env.step([_log("<retrieve>capital of france</retrieve>"), _log("no tool call")], [{}, {}])
    res = out.observations[0]["content"]
    assert res.startswith("<result>\n<1>\nthe capital of france is paris\n</1>") and "bananas" not in res
    assert out.observations[1]["content"] == "No retrieval query found!"
    assert out.next_stop_strings[0] == ["</retrieve>"] and out.rewards.sum() == 0
    # BM25 by hand for one term: idf(banana) = ln(1 + (3 - 1 + 0.5) / (1 + 0.5))
    r = env.retriever
    import math

    s = r.scores("bananas")
    avgdl = (6 + 4 + 6) / 3
    expect = math.log(1 + 2.5 / 1.5) * (1 * 2.5) / (1 + 1.5 * (1 - 0.75 + 0.75 * 4 / avgdl))
    assert s[1].item() == pytest.approx(expect, rel=1e-5) and s[0].item() == 0.0
