"""Rollout recovery ledger: lifecycle and state-dict rules, the rollout pump
serving in-flight groups before new prompts, and an async GRPO run resumed from
a checkpoint that regenerates the groups it had in flight (CPU)."""

from __future__ import annotations

import os
import time

import pytest
import torch

from rl_b200.algorithms.async_utils import AsyncTrajectoryCollector, ReplayBuffer
from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.experience.rollout_recovery import (GroupStatus, RolloutRecoveryLedger, collate_datums, datum_rows)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _datum(i):
    return {"message_log": [{"role": "user", "content": "", "token_ids": torch.arange(4) + i}], "length": 4,
            "extra_env_info": {"prompt_index": i}, "loss_multiplier": 1.0, "idx": i, "task_name": "t"}


def test_ledger_lifecycle_and_state_dict():
    led = RolloutRecoveryLedger()
    a = led.reserve_group(_datum(0), 2, target_step=0, weight_version=0)
    b = led.reserve_group(_datum(1), 2, target_step=1, weight_version=0)
    c = led.reserve_group(_datum(2), 2, target_step=1, weight_version=0)
    led.mark_dispatched(a)
    led.mark_group_sealed(a, [1.0, 0.0])
    led.mark_dispatched(b)
    led.mark_sibling_sealed(b, 0, 0.5)  # one sibling done, one still running
    assert led.counts() == {"reserved": 1, "dispatched": 1, "sealed": 1, "abandoned": 0}
    with pytest.raises(ValueError):
        led.mark_consumed([b])  # not sealed
    # failures: retried (back to reserved) until the attempt budget, then abandoned
    led.mark_dispatched(c)
    assert led.mark_failed(c, max_attempts=2) and led.get_group(c).status == GroupStatus.RESERVED
    led.mark_dispatched(c)
    assert not led.mark_failed(c, max_attempts=2) and led.get_group(c).status == GroupStatus.ABANDONED

    back = RolloutRecoveryLedger.from_state_dict(led.state_dict())
    assert back.state_dict() == led.state_dict()
    assert torch.equal(back.get_group(a).prompt["message_log"][0]["token_ids"], torch.arange(4))
    bad = led.state_dict()
    bad["groups"][0]["surprise"] = 1
    with pytest.raises(ValueError):
        RolloutRecoveryLedger.from_state_dict(bad)
    with pytest.raises(ValueError):
        RolloutRecoveryLedger.from_state_dict({**led.state_dict(), "schema_version": 99})

    # restart with the buffer holding group a: b (mid-generation) is redone with its
    # sealed sibling kept, a stays, c (abandoned) is not redone
    redo = back.prepare_for_restart(buffer_group_ids=[a])
    assert [g.group_id for g in redo] == [b] and back.get_group(b).unsealed_indices() == [1]
    # without a restored buffer the sealed group is regenerated too
    again = RolloutRecoveryLedger.from_state_dict(led.state_dict()).prepare_for_restart(None)
    assert [g.group_id for g in again] == [a, b]
    led.mark_consumed([a])
    assert a not in led and len(led) == 2


def test_datum_rows_round_trip():
    from rl_b200.data.datasets import rl_collate_fn

    rows = [_datum(i) for i in range(3)]
    batch = rl_collate_fn(rows)
    back = datum_rows(batch)
    assert [r["idx"] for r in back] == [0, 1, 2]
    again = collate_datums(back)
    assert torch.equal(again["length"], batch["length"]) and again["task_name"] == batch["task_name"]


def test_pump_serves_in_flight_groups_before_new_prompts():
    from rl_b200.data.datasets import rl_collate_fn

    old = RolloutRecoveryLedger()
    ids = [old.reserve_group(_datum(100 + i), 2, 0, 0) for i in range(2)]
    for gid in ids:
        old.mark_dispatched(gid)
    restart = old.prepare_for_restart(None)
    seen = []

    def rollout_fn(batch, target):
        seen.append([int(x) for x in batch["idx"]])
        rep = batch.repeat_interleave(2)
        rep["total_reward"] = torch.ones(len(rep["message_log"]))
        return rep, {}

    loader = [rl_collate_fn([_datum(0), _datum(1)]), rl_collate_fn([_datum(2), _datum(3)])]
    buf = ReplayBuffer(64)
    col = AsyncTrajectoryCollector(rollout_fn, loader, buf, num_prompt_groups=2, group_size=2,
                                   max_trajectory_age_steps=1, ledger=old, restart_groups=restart).start()
    t0 = time.time()
    while len(seen) < 2 and time.time() - t0 < 30:
        time.sleep(0.01)
    col.stop()
    col.check_health()
    assert seen[0] == [100, 101] and seen[1] == [0, 1]
    assert col.stats["groups_regenerated"] == 2
    sealed = [g for g in old.groups if g.status == GroupStatus.SEALED]
    assert {g.prompt_ref.sample_id for g in sealed} >= {100, 101, 0, 1}


def test_async_grpo_resume_regenerates_in_flight_groups(tmp_path):
    """Train 2 async steps with a checkpoint at step 2, drop the replay buffer on
    resume: the groups generated for later steps are regenerated from the ledger
    before the dataloader is asked for new prompts, and training completes."""
    from examples.run_grpo import main
    from rl_b200.algorithms.async_grpo import restore_rollout_recovery

    ck = str(tmp_path / "ckpt")
    common = ["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
              "logger.log_dir=" + str(tmp_path / "logs"), "logger.stdout=false",
              "++grpo.async_grpo.enabled=true", "++grpo.async_grpo.max_trajectory_age_steps=1",
              "++grpo.async_grpo.load_replay_buffer=false", "++loss_fn.use_importance_sampling_correction=true",
              "checkpointing.enabled=true", f"++checkpointing.checkpoint_dir={ck}", "++checkpointing.save_period=2"]
    state = main(common + ["grpo.max_num_steps=2"])
    assert state["current_step"] == 2
    step_dir = os.path.join(ck, "step_2")
    led = restore_rollout_recovery(step_dir)
    assert led is not None
    pending = [g for g in led.groups if g.status != GroupStatus.ABANDONED]
    assert pending, "the pump had groups beyond step 2 in flight or buffered"
    logs2 = str(tmp_path / "logs2")
    state = main([a if not a.startswith("logger.log_dir=") else "logger.log_dir=" + logs2 for a in common]
                 + ["grpo.max_num_steps=3"])
    assert state["current_step"] == 3
    import json

    with open(os.path.join(logs2, "metrics.jsonl")) as f:
        rows = [json.loads(line) for line in f]
    regen = [r["train/groups_regenerated"] for r in rows if "train/groups_regenerated" in r]
    assert regen and regen[-1] >= len(pending)
