"""Forest training rows (context compaction / retries / branches): the
worked examples of the reference's guide, once-only loss ownership and the
per-owner advantage broadcast."""

import pytest
import torch

from rl_b200.algorithms.advantage_estimator import make_advantage_estimator
from rl_b200.experience.forest import (CapturedCall, fanout, owner_advantages, reconstruct_rows, rollout_rows,
                                       select_calls)


def C(cid, parent, inp, out, **kw):
    return CapturedCall(cid, parent, list(inp), list(out), [-0.1 * (i + 1) for i in range(len(out))], **kw)


def test_chain_is_one_row():
    calls = [C("c1", None, [1, 2], [10, 11]), C("c2", "c1", [3], [12]), C("c3", "c2", [4], [13, 14])]
    rows, ok = rollout_rows(calls, returned_ids=["c1", "c2", "c3"], terminal_id="c3")
    assert ok and len(rows) == 1
    r = rows[0]
    assert r.token_ids.tolist() == [1, 2, 10, 11, 3, 12, 4, 13, 14]
    assert r.token_loss_mask.tolist() == [0, 0, 1, 1, 0, 1, 0, 1, 1]
    assert r.generation_logprobs.tolist()[2:4] == pytest.approx([-0.1, -0.2])


def test_rewrite_rejected_retry_give_two_rows():
    # c1 -> c2 accepted; the harness compacts: c3 is a new root; c4 rejected, c5 retries from c3
    calls = [C("c1", None, [1, 2], [10]), C("c2", "c1", [3], [11]), C("c3", None, [9, 9], [12]),
             C("c4", "c3", [4], [13]), C("c5", "c3", [4], [14])]
    rows, ok = rollout_rows(calls, returned_ids=["c1", "c2", "c3", "c5"], terminal_id="c5")
    assert ok and [r.call_ids for r in rows] == [["c1", "c2"], ["c3", "c5"]]
    assert rows[1].token_ids.tolist() == [9, 9, 12, 4, 14]
    assert rows[1].token_loss_mask.tolist() == [0, 0, 1, 0, 1]  # rewritten prompt is context only


def test_shared_ancestor_trains_once():
    calls = [C("a", None, [1], [10, 11]), C("b", "a", [2], [12]), C("c", "a", [3], [13])]
    sel = select_calls(calls, "all_captured", terminal_id="c")
    rows = reconstruct_rows(calls, sel)
    assert [r.call_ids for r in rows] == [["a", "b"], ["a", "c"]]
    assert rows[0].token_loss_mask.tolist() == [0, 1, 1, 0, 1]
    assert rows[1].token_loss_mask.tolist() == [0, 0, 0, 0, 1]  # a is context in the second path
    total = sum(float(r.token_loss_mask.sum()) for r in rows)
    assert total == 4  # every generated token once


def test_selection_rules():
    calls = [C("a", None, [1], [10]), C("b", "a", [2], [11]), C("x", "a", [2], [12], status="failed"),
             C("y", "b", [3], [13], status="incomplete", finish_reason="content_filter"),
             C("z", "b", [3], [14], status="incomplete", finish_reason="length")]
    assert select_calls(calls, "all_captured", terminal_id="z") == ["a", "b", "z"]
    with pytest.raises(ValueError, match="omits"):
        select_calls(calls, "returned_history", returned_ids=["b"])
    with pytest.raises(ValueError, match="never captured"):
        select_calls(calls, "returned_history", returned_ids=["a", "q"])
    with pytest.raises(ValueError, match="scored call"):
        select_calls(calls, "returned_history", returned_ids=["a"], terminal_id="b")
    # a kept failed call masks the rollout
    calls2 = [C("a", None, [1], [10]), C("b", "a", [2], [11], status="failed")]
    _, ok = rollout_rows(calls2, returned_ids=["a", "b"], terminal_id="b")
    assert not ok


def test_owner_advantage_fanout():
    est = make_advantage_estimator({"name": "grpo", "normalize_rewards": False, "use_leave_one_out_baseline": False})
    rewards = torch.tensor([1.0, 0.0, 1.0, 0.0])  # two prompt groups of two rollouts
    gid = torch.tensor([0, 0, 1, 1])
    adv = owner_advantages(est, gid, rewards)
    assert adv.tolist() == [0.5, -0.5, 0.5, -0.5]
    # owner 0 was split into three rows, owner 1 into one; -1 is execution padding
    row_owner = torch.tensor([0, 0, 0, 1, 2, 3, -1])
    assert fanout(adv, row_owner).tolist() == [0.5, 0.5, 0.5, -0.5, 0.5, -0.5, 0.0]
    adv = owner_advantages(est, gid, rewards, valid=torch.tensor([1.0, 1.0, 1.0, 0.0]))
    assert adv.tolist() == [0.5, -0.5, 0.0, 0.0]
