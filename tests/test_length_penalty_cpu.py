"""``grpo.length_penalty`` against golden vectors of the reference's
``apply_group_length_penalties`` (``tests/data/length_penalty_goldens.json``:
inputs, configs and expected rewards / metrics; lengths in characters), plus
config validation and the GRPO rollout hook."""

import json
import math
import os

import pytest
import torch

from rl_b200.algorithms.length_penalty import (LengthPenaltyConfig, apply_group_length_penalties,
                                               apply_length_penalty_to_rollout, split_reasoning_answer)

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "data", "length_penalty_goldens.json")))


def _rows(case):
    rows = []
    for r in case["rows"]:
        out = []
        if r["reasoning_chars"]:
            out.append({"type": "reasoning", "summary": [{"text": "x" * r["reasoning_chars"]}]})
        out.append({"type": "message", "role": "assistant", "content": [{"text": "y" * r["answer_chars"]}]})
        row = {"reward": r["reward"], "agent": r["agent"], "response": {"output": out},
               "generated_tokens": r["generated_tokens"]}
        for k in ("profiled_rewards", "profiled_output_lengths", "profile_band"):
            if k in r:
                row[k] = r[k]
        rows.append(row)
    return rows


@pytest.mark.parametrize("ci", range(len(GOLD["cases"])))
def test_matches_reference_goldens(ci):
    case = GOLD["cases"][ci]
    rows = _rows(case)
    m = apply_group_length_penalties(rows, case["config"], case["group_size"])
    got = [r["reward"] for r in rows]
    for g, e in zip(got, case["expected_rewards"]):
        assert math.isclose(g, e, rel_tol=1e-9, abs_tol=1e-12), (got, case["expected_rewards"])
    for k, v in case["expected_metrics"].items():
        assert math.isclose(m[k], v, rel_tol=1e-9, abs_tol=1e-12), (k, m[k], v)


def test_config_validation():
    with pytest.raises(ValueError, match="unknown"):
        LengthPenaltyConfig({"default": {"total_bonsu": 0.1}})
    with pytest.raises(ValueError, match="length_type"):
        LengthPenaltyConfig({"default": {"length_type": "words"}})
    with pytest.raises(ValueError, match="b > a"):
        LengthPenaltyConfig({"profile_band": {"enabled": True, "defaults": {"total": {"a": 5, "b": 5, "f": 0.5}}}})
    with pytest.raises(ValueError, match=r"\[0, 1\]"):
        LengthPenaltyConfig({"profile_band": {"enabled": True, "defaults": {"total": {"a": 5, "b": 9, "f": 1.5}}}})
    with pytest.raises(ValueError, match="zero_over_max"):
        LengthPenaltyConfig({"default": {"profiled_length_penalty_type": "zero_over_max",
                                         "profiled_length_penalty": 0.2}})
    with pytest.raises(ValueError, match="only applies to zero_over_max"):
        LengthPenaltyConfig({"default": {"profiled_length_allow_non_binary_rewards": True}})
    with pytest.raises(ValueError, match="all_generated_tokens"):
        LengthPenaltyConfig({"default": {"length_type": "all_generated_tokens", "reasoning_bonus": 0.1}})
    # an override that is fine alone but not merged with the default
    with pytest.raises(ValueError, match="agent 'x'"):
        LengthPenaltyConfig({"default": {"profiled_length_penalty_type": "zero_over_max"},
                             "agent_overrides": {"x": {"profiled_length_penalty": 0.2}}})
    cfg = LengthPenaltyConfig({"profile_band": {"enabled": True, "defaults": {"total": {"a": 1, "b": 2, "f": 0.5}}},
                               "default": {"profile_band_total": False}})
    assert cfg.default["profile_band_total"] is False
    cfg = LengthPenaltyConfig({"profile_band": {"enabled": True, "defaults": {"total": {"a": 1, "b": 2, "f": 0.5}}}})
    assert cfg.default["profile_band_total"] is True


def test_profiled_fields_required():
    rows = [{"reward": 1.0, "agent": "a", "message_log": [{"role": "assistant", "content": "abc"}]}] * 2
    with pytest.raises(ValueError, match="profiled_rewards"):
        apply_group_length_penalties([dict(r) for r in rows], {"default": {"profiled_length_penalty": 0.1}}, 2)


def test_think_split_and_observations_ignored():
    log = [{"role": "user", "content": "q"},
           {"role": "assistant", "content": "<think>abcd</think>xyz"},
           {"role": "environment", "content": "observation text"},
           {"role": "assistant", "content": "<think>ef</think>uv"}]
    assert split_reasoning_answer({"message_log": log}) == ("abcdef", "xyzuv")


def test_rollout_hook_keeps_env_reward():
    G = 4
    logs = [[{"role": "user", "content": "q", "token_ids": torch.zeros(3, dtype=torch.long)},
             {"role": "assistant", "content": "<think>" + "t" * (10 * (k + 1)) + "</think>ans",
              "token_ids": torch.zeros(5, dtype=torch.long)}] for k in range(G)]
    rollout = {"message_log": logs, "total_reward": torch.tensor([1.0, 1.0, 0.0, 1.0]),
               "extra_env_info": [{"agent_ref": {"name": "math"}}] * G, "task_name": ["math"] * G}
    m = apply_length_penalty_to_rollout(rollout, {"default": {"group_total_length_penalty_coeff": 0.3}}, G)
    assert torch.equal(rollout["env_reward"], torch.tensor([1.0, 1.0, 0.0, 1.0]))
    r = rollout["total_reward"]
    assert r[0] > 1.0 > r[3] and r[2] == 0.0 and abs(float(r[[0, 1, 3]].mean()) - 1.0) < 1e-6
    assert m["length_penalty/adjusted_frac"] == 0.75 and m["length_penalty/env_reward_mean"] == 0.75
    # agent disabled under agent_overrides: untouched
    rollout["total_reward"] = rollout["env_reward"].clone()
    m = apply_length_penalty_to_rollout(rollout, {"default": {"group_total_length_penalty_coeff": 0.3},
                                                  "agent_overrides": {"math": {"enabled": False}}}, G)
    assert torch.equal(rollout["total_reward"], rollout["env_reward"]) and m["length_penalty/adjusted_frac"] == 0.0


def test_grpo_loop_with_length_penalty(tmp_path):
    """A tiny GRPO run with ``grpo.length_penalty`` set logs its metrics."""
    import glob

    from examples.run_grpo import main

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    state = main(["--config", os.path.join(root, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  f"logger.log_dir={tmp_path}", "logger.stdout=false",
                  "++grpo.length_penalty.default.group_total_length_penalty_coeff=0.1",
                  "++grpo.length_penalty.default.length_type=chars"])
    assert state["current_step"] == 2
    text = "".join(open(f).read() for f in glob.glob(str(tmp_path / "**" / "*"), recursive=True)
                   if os.path.isfile(f))
    assert "length_penalty/env_reward_mean" in text
