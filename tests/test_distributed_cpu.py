"""Tensor / sequence / data / expert parallelism on CPU gloo ranks, each compared with
a single-process run of the same step (same seed, same global batch).

Mirrors the reference's distributed unit-test strategy (spawned localhost ranks
compared against a single-device baseline, ``tests/unit/distributed/test_distributed_logprob.py``)."""

import pytest
import torch

from rl_b200.distributed.launch import spawn_ranks
from tests.dist_cases import case_train_step


@pytest.fixture(scope="module")
def dense_single():
    return spawn_ranks(case_train_step, 1, 1, 1, False, False)[0]


@pytest.fixture(scope="module")
def moe_single():
    return spawn_ranks(case_train_step, 1, 1, 1, False, True)[0]


def _close(a, b, tol=2e-4):
    assert abs(a["loss"] - b["loss"]) < tol * max(1.0, abs(b["loss"])), (a["loss"], b["loss"])
    assert abs(a["grad_norm"] - b["grad_norm"]) < tol * max(1.0, b["grad_norm"]), (a["grad_norm"], b["grad_norm"])
    assert torch.allclose(a["lp"], b["lp"], atol=5e-4), (a["lp"] - b["lp"]).abs().max()


@pytest.mark.parametrize("world,tp,sp", [(2, 2, False), (2, 2, True), (2, 1, False), (4, 2, False), (4, 2, True)])
def test_dense_parallel_matches_single(dense_single, world, tp, sp):
    outs = spawn_ranks(case_train_step, world, tp, 1, sp, False)
    for o in outs:
        _close(o, dense_single)


def test_moe_expert_parallel_matches_single(moe_single):
    outs = spawn_ranks(case_train_step, 2, 1, 2, False, True)
    for o in outs:
        _close(o, moe_single)


def test_reshard_refit_tp2_to_rollout_tp1():
    from tests.dist_cases import case_reshard_refit

    outs = spawn_ranks(case_reshard_refit, 2, 2)
    for o in outs:
        assert o["init_err"] == 0.0, o["init_err"]
        assert o["refit_err"] == 0.0, o["refit_err"]
    assert torch.equal(outs[0]["out_ids"], outs[1]["out_ids"])
    assert outs[0]["out_ids"].shape[0] == 5


@pytest.mark.parametrize("world,tp,cp,sp", [(2, 1, 2, False), (4, 2, 2, True), (4, 1, 2, False)])
def test_context_parallel_matches_single(dense_single, world, tp, cp, sp):
    """Load-balanced CP chunks + gathered-KV attention reproduce the single-process step."""
    outs = spawn_ranks(case_train_step, world, tp, 1, sp, False, cp)
    for o in outs:
        _close(o, dense_single)
