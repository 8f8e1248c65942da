"""Async GRPO pieces on CPU: replay-buffer targeting / staleness rules, the
rollout pump's target reservation, the split train API against ``train``, and
an end-to-end async run of the tiny config."""

import os
import threading

import pytest
import torch

from rl_b200.algorithms.async_utils import AsyncTrajectoryCollector, ReplayBuffer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_replay_buffer_targets_and_staleness():
    rb = ReplayBuffer(max_size=6)
    for i in range(2):
        assert rb.add(("a", i), weight_version=0, target_weight_version=0) == "success"
    rb.add(("b", 0), 0, 1)
    assert rb.sample(3, current_weight_version=0, max_age_steps=1) is None  # only 2 meant for step 0
    s = rb.sample(2, 0, 1)
    assert [g for g in s["trajectories"]] == [("a", 0), ("a", 1)] and s["avg_trajectory_age"] == 0
    assert rb.size() == 1 and rb.last_consumed_target == 0
    rb.add(("b", 1), 1, 1)
    s = rb.sample(2, 1, 1)
    assert s["avg_trajectory_age"] == 0.5
    # stale groups (generated more than max_age updates ago) are evicted
    rb.add(("c", 0), 0, 3)
    assert rb.sample(1, 3, 1) is None and rb.size() == 0
    for i in range(6):
        rb.add(i, 3, 4)
    assert rb.add(99, 3, 4) == "full"
    sd = rb.state_dict()
    rb2 = ReplayBuffer(6)
    rb2.load_state_dict(sd, drop_incomplete_targets=7)
    assert rb2.size() == 0
    rb2.load_state_dict(sd)
    assert rb2.size() == 6 and rb2.has_complete_batch(4, 6)


def test_collector_reserves_targets_within_lead():
    rb = ReplayBuffer(100)
    c = AsyncTrajectoryCollector(None, [], rb, num_prompt_groups=2, group_size=1, max_trajectory_age_steps=2)
    assert c.target_candidates(0) == [0, 1, 2]
    assert c.target_candidates(3) == [4, 5]
    assert c._reserve_target(0) == 0 and c._reserve_target(0) == 1 and c._reserve_target(0) == 2
    assert c._reserve_target(0) is None  # every target in the window is being generated
    c._generating.clear()
    rb.add("x", 0, 0)
    rb.add("y", 0, 0)
    assert c._reserve_target(0) == 1  # target 0 already complete


def test_split_train_api_matches_train():
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from tests.dist_cases import make_batch
    from tests.test_core_cpu import _tiny_policy

    data = make_batch(B=8, S=24, seed=3)
    lf = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    a = _tiny_policy(seed=1)
    ra = a.train(data, lf, gbs=8)
    b = _tiny_policy(seed=1)
    st = b.begin_train_step(data, lf)
    assert st.num_microbatches >= 2
    for i in range(st.num_microbatches):
        b.train_microbatch(st, i)
    rb_ = b.finish_train_step(st)
    assert abs(ra["loss"] - rb_["loss"]) < 1e-6 and abs(ra["grad_norm"] - rb_["grad_norm"]) < 1e-5
    assert torch.equal(a.model.flat_param, b.model.flat_param)
    st = b.begin_train_step(data, lf)
    with pytest.raises(RuntimeError):
        b.finish_train_step(st)


def test_async_grpo_tiny_runs():
    from examples.run_grpo import main

    state = main(["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  "logger.log_dir=/tmp/rlb_test_logs_async", "logger.stdout=false",
                  "grpo.max_num_steps=3", "++grpo.async_grpo.enabled=true",
                  "++grpo.async_grpo.max_trajectory_age_steps=1",
                  "++loss_fn.use_importance_sampling_correction=true"])
    assert state["current_step"] == 3
    # no pump thread is left behind
    assert not [t for t in threading.enumerate() if t.name == "rollout-pump" and t.is_alive()]


def test_replay_buffer_checkpoint_file_round_trip(tmp_path):
    """The async loop's replay buffer is written per rank into the checkpoint
    directory and restored from it (incomplete targets dropped); restoring is
    skipped when disabled or when the file is absent."""
    from rl_b200.algorithms.async_grpo import replay_buffer_file, restore_replay_buffer
    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    rb = ReplayBuffer(8)
    for tgt in (3, 3, 4):
        rb.add(BatchedDataDict({"x": torch.arange(3) + tgt}), weight_version=2, target_weight_version=tgt)
    torch.save(rb.state_dict(), tmp_path / replay_buffer_file())
    back = restore_replay_buffer(str(tmp_path), num_prompt_groups=2, max_size=8)
    assert back is not None and back.existing_targets() == {3} and back.count_for_target(3) == 2
    assert restore_replay_buffer(str(tmp_path), 2, 8, load_replay_buffer=False) is None
    assert restore_replay_buffer(str(tmp_path / "missing"), 2, 8) is None
