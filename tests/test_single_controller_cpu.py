"""SingleController: pumps, back-pressure, trajectory age, per-prompt failure
budgets with backoff, dropped-prompt policies, the stall watchdog, lockstep step
sizes over gloo ranks, and GRPO through the controller on the tiny model (CPU)."""

from __future__ import annotations

import os
import threading
import time

import pytest
import torch

from rl_b200.algorithms.single_controller import RolloutDataError, SingleController, StallError
from rl_b200.distributed.batched_data_dict import BatchedDataDict

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _loader(n_prompts: int, per_batch: int = 2):
    """A dataloader of prompt batches in the collated datum layout."""
    rows = [{"message_log": [{"role": "user", "content": f"p{i}", "token_ids": torch.tensor([i, i + 1])}],
             "task_name": "t", "extra_env_info": {"i": i}, "length": 2, "loss_multiplier": 1.0, "idx": i}
            for i in range(n_prompts)]
    from rl_b200.experience.rollout_recovery import collate_datums

    return [collate_datums(rows[i:i + per_batch]) for i in range(0, n_prompts, per_batch)]


def _fake_generate(log: list, fail=None, delay_s: float = 0.0):
    def gen(batch, version):
        idx = [int(x) for x in batch["idx"]]
        if fail is not None:
            fail(idx)
        if delay_s:
            time.sleep(delay_s)
        log.append((version, sorted(set(idx))))
        n = len(idx)
        logs = [[dict(m) for m in batch["message_log"][i]] + [{"role": "assistant", "content": "a",
                                                               "token_ids": torch.tensor([7])}] for i in range(n)]
        return BatchedDataDict({"message_log": logs, "idx": torch.tensor(idx), "task_name": list(batch["task_name"]),
                                "total_reward": torch.ones(n), "version": torch.full((n,), version)})
    return gen


def _fake_train(seen: list, delay_s: float = 0.0):
    def train(groups, version):
        if delay_s:
            time.sleep(delay_s)
        seen.append((version, [int(g["idx"][0]) for g in groups], [int(g["version"][0]) for g in groups]))
        return {"loss": 0.0}
    return train


def test_pumps_train_every_step_with_full_groups_and_bounded_age():
    gens, seen = [], []
    sc = SingleController(_fake_generate(gens), _fake_train(seen, delay_s=0.01), _loader(32), group_size=4,
                          groups_per_step=4, max_steps=5,
                          cfg={"max_inflight_prompts": 2, "max_buffered_rollouts": 6}, max_trajectory_age_steps=1)
    hist = sc.run()
    assert len(hist) == 5 and [len(s[1]) for s in seen] == [4] * 5
    for version, _, gen_versions in seen:
        assert all(version - 1 <= v <= version for v in gen_versions)  # age <= 1
    assert max(len(ix) for _, ix in gens) <= 2                            # one call <= max_inflight_prompts
    trained = [i for _, ix, _ in seen for i in ix]
    assert len(trained) == len(set(trained))                             # every group trained once
    assert all(h["groups"] == 4.0 for h in hist)


def test_stale_groups_are_evicted_and_regenerated():
    gens, seen = [], []
    # generation is fast and the trainer slow: with age 0 a buffered group is stale after a step
    sc = SingleController(_fake_generate(gens), _fake_train(seen, delay_s=0.05), _loader(64), group_size=2,
                          groups_per_step=2, max_steps=4, cfg={"max_inflight_prompts": 2, "max_buffered_rollouts": 6},
                          max_trajectory_age_steps=0)
    sc.run()
    assert sc.stats["groups_evicted"] > 0
    for version, _, gen_versions in seen:
        assert all(v == version for v in gen_versions)
    regenerated = [i for _, ix in gens for i in ix]
    assert len(regenerated) > len(set(regenerated))  # evicted prompts came back


def test_infra_failures_retry_with_backoff_then_succeed():
    gens, seen = [], []
    calls = {"n": 0}

    def fail(idx):
        calls["n"] += 1
        if 3 in idx and calls["n"] <= 3:
            raise RuntimeError("engine died")

    sc = SingleController(_fake_generate(gens, fail), _fake_train(seen), _loader(8), group_size=2,
                          groups_per_step=2, max_steps=4,
                          cfg={"max_inflight_prompts": 2,
                               "rollout_failure": {"backoff_base_s": 0.01, "max_backoff_s": 0.02,
                                                   "max_infra_attempts_per_prompt": 5}})
    sc.run()
    assert sc.stats["infra_failures"] >= 1 and sc.stats["retries"] >= 2 and sc.stats["prompts_skipped"] == 0
    assert 3 in [i for _, ix, _ in seen for i in ix]


def test_data_failures_drop_the_prompt_and_shrink_the_step():
    gens, seen = [], []

    def fail(idx):
        if 5 in idx:
            raise RolloutDataError("prompt cannot be rendered")

    sc = SingleController(_fake_generate(gens, fail), _fake_train(seen), _loader(8, per_batch=1), group_size=2,
                          groups_per_step=4, max_steps=2,
                          cfg={"max_inflight_prompts": 1,
                               "rollout_failure": {"backoff_base_s": 0.0, "max_data_attempts_per_prompt": 2,
                                                   "max_skipped_prompts": 1, "min_step_batch_fraction": 0.75,
                                                   "on_dropped_prompt": "shrink"}})
    sc.run()
    assert sc.stats["data_failures"] == 2 and sc.stats["prompts_skipped"] == 1
    assert 5 not in [i for _, ix, _ in seen for i in ix]
    assert sc.stats["shrunk_steps"] >= 1 and min(len(ix) for _, ix, _ in seen) == 3


def test_too_many_skipped_prompts_end_the_run():
    def fail(idx):
        raise RolloutDataError("bad")

    sc = SingleController(_fake_generate([], fail), _fake_train([]), _loader(8), group_size=2, groups_per_step=2,
                          max_steps=2, cfg={"rollout_failure": {"backoff_base_s": 0.0, "max_skipped_prompts": 0,
                                                                "max_data_attempts_per_prompt": 1}})
    with pytest.raises(RuntimeError, match="max_skipped_prompts"):
        sc.run()


def test_watchdog_aborts_a_stalled_generation_and_warns_otherwise():
    wd = {"interval_s": 0.05, "stall_timeout_s": 0.3}
    sc = SingleController(_fake_generate([], delay_s=1.5), _fake_train([]), _loader(8), group_size=2,
                          groups_per_step=2, max_steps=2, cfg={"stall_watchdog": {**wd, "stall_action": "abort"}})
    t0 = time.perf_counter()
    with pytest.raises(StallError, match="rollout"):
        sc.run()
    assert time.perf_counter() - t0 < 1.4  # ended by the watchdog, before the call returned
    sc = SingleController(_fake_generate([], delay_s=0.5), _fake_train([]), _loader(8), group_size=2,
                          groups_per_step=2, max_steps=1, cfg={"stall_watchdog": {**wd, "stall_action": "warn"}})
    assert len(sc.run()) == 1 and sc.stats["stalls"] >= 1


def test_back_pressure_bounds_buffered_groups():
    peak = {"n": 0}
    sc = None

    def fail(idx):
        peak["n"] = max(peak["n"], len(sc._ready))

    sc = SingleController(_fake_generate([], fail), _fake_train([], delay_s=0.05), _loader(40), group_size=2,
                          groups_per_step=2, max_steps=4, cfg={"max_inflight_prompts": 2, "max_buffered_rollouts": 4},
                          max_trajectory_age_steps=8)
    sc.run()
    assert peak["n"] <= 4


def test_controller_state_round_trip():
    sc = SingleController(_fake_generate([]), _fake_train([]), _loader(8), group_size=2, groups_per_step=2,
                          max_steps=1)
    sc.run()
    sd = sc.state_dict()
    sc2 = SingleController(_fake_generate([]), _fake_train([]), _loader(8), group_size=2, groups_per_step=2,
                           max_steps=1)
    sc2.load_state_dict(sd)
    assert sc2.version == sc.version and set(sc2._ready) == set(sc._ready)


def test_data_parallel_ranks_agree_on_step_sizes():
    from rl_b200.distributed.launch import spawn_ranks
    from tests.dist_cases import case_single_controller_dp

    a, b = spawn_ranks(case_single_controller_dp, 2)
    assert a == b and len(a) == 2


def test_grpo_through_the_single_controller(tmp_path):
    from examples.run_grpo import main

    state = main(["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  "logger.log_dir=" + str(tmp_path / "logs"), "logger.stdout=false",
                  "++grpo.single_controller.enabled=true", "++grpo.single_controller.max_inflight_prompts=4"])
    assert state["current_step"] == 2 and state["single_controller"]["groups_generated"] >= 16


def test_controller_keeps_the_rollout_ledger():
    """With a recovery ledger every trained group is consumed, a dropped prompt is
    forgotten, and nothing stays in flight after the run."""
    from rl_b200.experience.rollout_recovery import RolloutRecoveryLedger

    def fail(idx):
        if 1 in idx:
            raise RolloutDataError("bad")

    ledger = RolloutRecoveryLedger()
    sc = SingleController(_fake_generate([], fail), _fake_train([]), _loader(6, per_batch=1), group_size=2,
                          groups_per_step=2, max_steps=2, ledger=ledger,
                          cfg={"max_inflight_prompts": 1,
                               "rollout_failure": {"backoff_base_s": 0.0, "max_data_attempts_per_prompt": 1,
                                                   "max_skipped_prompts": 1}})
    sc.run()
    groups = ledger.groups
    sealed = [g for g in groups if g.status.value == "sealed"]
    # trained groups were consumed; what remains is buffered (sealed) or was in flight at the end
    assert len(sealed) == len(sc._ready), (len(sealed), len(sc._ready))
    assert {g.status.value for g in groups} <= {"sealed", "dispatched", "reserved"}
    assert all(int(g.prompt.get("idx", -1)) != 1 for g in groups)  # the dropped prompt was forgotten
