"""Sharding / micro-batch planning behaviour of ``BatchedDataDict`` and the
packers' bin-count constraints (reference: ``tests/unit/distributed/
test_batched_data_dict.py`` and ``tests/unit/data/packing/test_algorithms.py``)."""

import random

import pytest
import torch

from rl_b200.data.packing import BalancedGreedyKnapsackPacker, GreedyKnapsackPacker, get_packer
from rl_b200.distributed.batched_data_dict import BatchedDataDict

ALGS = ["concatenative", "first_fit", "first_fit_decreasing", "first_fit_shuffle", "modified_first_fit_decreasing",
        "greedy_knapsack", "balanced_greedy_knapsack"]


def _batch(lengths, width=100):
    lengths = torch.tensor(lengths)
    return BatchedDataDict({"input_ids": torch.ones(len(lengths), width, dtype=torch.long),
                            "sequence_lengths": lengths, "problem_ids": torch.arange(len(lengths))})


def _pack_args(order=None, cap=100, **kw):
    a = {"max_tokens_per_microbatch": cap, "input_key": "input_ids", "input_lengths_key": "sequence_lengths",
         "algorithm": "modified_first_fit_decreasing", "sequence_length_pad_multiple": 1}
    if order is not None:
        a["microbatch_order"] = order
    a.update(kw)
    return a


def test_packed_bins_round_robin_largest_first():
    d = _batch([46, 24, 55, 88, 11, 14, 73, 17])
    packer_shards, _ = d.shard_by_batch_size(2, sequence_packing_args=_pack_args("packer"))
    shards, order = d.shard_by_batch_size(2, sequence_packing_args=_pack_args("largest_first"))
    assert [s.micro_batch_lengths[0] for s in shards] == [[99, 96], [87, 46]]
    for p, q in zip(packer_shards, shards):
        assert set(p["problem_ids"].tolist()) == set(q["problem_ids"].tolist())
        assert sorted(p.micro_batch_lengths[0], reverse=True) == q.micro_batch_lengths[0]
    back = BatchedDataDict.from_batches(shards)
    back.reorder_data(order)
    assert torch.equal(back["problem_ids"], d["problem_ids"])
    assert torch.equal(back["sequence_lengths"], d["sequence_lengths"])


def test_unknown_microbatch_order_rejected():
    d = _batch([4, 5], width=8)
    with pytest.raises(ValueError, match="microbatch_order"):
        d.shard_by_batch_size(1, sequence_packing_args=_pack_args("unknown", cap=8))


def test_largest_first_keeps_chunk_boundaries():
    d = _batch([46, 24, 55, 88, 11, 14, 73, 17, 31, 67, 19, 82, 12, 43, 58, 21])
    shards, order = d.shard_by_batch_size(2, batch_size=8, sequence_packing_args=_pack_args("largest_first"))
    for sh in shards:
        assert len(sh.micro_batch_lengths) == 2
        for lens in sh.micro_batch_lengths:
            assert lens == sorted(lens, reverse=True)
        n0, n1 = sh.elem_counts_per_gb
        assert torch.all(sh["problem_ids"][:n0] < 8) and torch.all(sh["problem_ids"][n0:n0 + n1] >= 8)
        gb1 = sh.get_batch(1)
        assert gb1.size == n1 and torch.all(gb1["problem_ids"] >= 8)
        assert sum(m.size for m in gb1.make_microbatch_iterator_for_packable_sequences()) == n1
    back = BatchedDataDict.from_batches(shards)
    back.reorder_data(order)
    assert torch.equal(back["problem_ids"], d["problem_ids"])


def test_uniform_lengths_pack_evenly():
    d = _batch([256] * 16, width=256)
    shards, _ = d.shard_by_batch_size(2, sequence_packing_args=_pack_args(cap=1024))
    counts = [s.get_microbatch_iterator_for_packable_sequences_len()[0] for s in shards]
    assert sum(counts) == 4 and min(counts) == 2
    for s in shards:
        assert all(L <= 1024 for L in s.micro_batch_lengths[0])


def test_pair_grouping_keeps_pairs_together():
    rng = random.Random(1)
    lens = [rng.randint(5, 40) for _ in range(16)]
    d = _batch(lens)
    d["pair"] = torch.arange(16) // 2
    shards, order = d.shard_by_batch_size(2, sequence_packing_args=_pack_args(cap=100, pair_grouping_key="pair"))
    for sh in shards:
        for mb in sh.make_microbatch_iterator_for_packable_sequences():
            pairs = mb["pair"].tolist()
            assert all(pairs.count(p) == 2 for p in pairs)
    with pytest.raises(KeyError):
        d.shard_by_batch_size(2, sequence_packing_args=_pack_args(pair_grouping_key="nope"))


def test_dynamic_batching_same_plan_every_shard():
    rng = random.Random(0)
    lens = [rng.randint(3, 60) for _ in range(32)]
    d = _batch(lens, width=64)
    args = {"max_tokens_per_microbatch": 128, "sequence_length_round": 8, "input_key": "input_ids",
            "input_lengths_key": "sequence_lengths"}
    shards, order = d.shard_by_batch_size(4, batch_size=16, dynamic_batching_args=args)
    assert all(s.micro_batch_indices == shards[0].micro_batch_indices for s in shards)
    assert all(s.micro_batch_lengths == shards[0].micro_batch_lengths for s in shards)
    # each shard holds 4 rows of each chunk, chunk by chunk, dealt by length
    for sh in shards:
        assert torch.all(sh["problem_ids"][:4] < 16) and torch.all(sh["problem_ids"][4:] >= 16)
    firsts = [int(sh["sequence_lengths"][:4].min()) for sh in shards]
    assert max(firsts) <= sorted(lens[:16])[3]
    for sh in shards:
        n = 0
        for mb in sh.make_microbatch_iterator_with_dynamic_shapes():
            assert mb["input_ids"].shape[1] * mb.size <= 128
            assert int(mb["sequence_lengths"].max()) <= mb["input_ids"].shape[1]
            n += mb.size
        assert n == sh.size
    assert shards[0].get_microbatch_iterator_dynamic_shapes_len() == sum(len(c) for c in shards[0].micro_batch_indices)
    back = BatchedDataDict.from_batches(shards)
    back.reorder_data(order)
    assert torch.equal(back["problem_ids"], d["problem_ids"])


@pytest.mark.parametrize("alg", ALGS)
def test_packer_min_and_multiple_bins(alg):
    rng = random.Random(3)
    lens = [rng.randint(10, 60) for _ in range(30)]
    natural = len(get_packer(alg, 100).pack(lens))
    more = get_packer(alg, 100, min_bin_count=natural + 2).pack(lens)
    assert len(more) == natural + 2 and all(more)
    forced = get_packer(alg, 100, min_bin_count=natural + 1, bin_count_multiple=4).pack(lens)
    assert len(forced) % 4 == 0 and len(forced) >= natural + 1
    for bins in (more, forced):
        assert sorted(i for b in bins for i in b) == list(range(30))
        assert all(sum(lens[i] for i in b) <= 100 for b in bins)


@pytest.mark.parametrize("alg", ALGS)
def test_packer_item_cap(alg):
    lens = [5] * 20
    bins = get_packer(alg, 100, max_sequences_per_bin=3).pack(lens)
    assert all(len(b) <= 3 for b in bins) and sorted(i for b in bins for i in b) == list(range(20))


def test_packer_constraint_errors():
    with pytest.raises(ValueError):
        get_packer("concatenative", 100, min_bin_count=-1)
    with pytest.raises(ValueError):
        get_packer("concatenative", 100, bin_count_multiple=0)
    with pytest.raises(ValueError, match="Cannot create 3 bins with only 2 sequences"):
        get_packer("concatenative", 100, min_bin_count=3).pack([50, 50])
    with pytest.raises(ValueError, match="Cannot create 4 bins with only 2 sequences"):
        get_packer("concatenative", 100, bin_count_multiple=4).pack([50, 50])


def test_balanced_knapsack_delta():
    assert BalancedGreedyKnapsackPacker(8, balanced_knapsack_delta=0).pack([4, 4, 4, 4]) == [[0, 2], [1, 3]]
    assert get_packer("balanced_greedy_knapsack", 8, balanced_knapsack_delta=1).pack([4, 4, 4, 4]) == [[0, 3], [1], [2]]
    for p in (GreedyKnapsackPacker(10), BalancedGreedyKnapsackPacker(10)):
        p.max_sequences_per_bin = 1
        assert p.pack([4, 3, 2]) == [[0], [1], [2]]
        with pytest.raises(ValueError, match="exceeds bin capacity"):
            p.pack([11])


def test_worker_largest_first_and_item_cap():
    """``policy.sequence_packing.microbatch_order`` / ``max_sequences_per_bin``
    reach the policy worker's packing plan; the loss does not depend on the
    micro-batch order."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY, _pcfg, make_batch

    losses = []
    for order in ("packer", "largest_first"):
        cfg = _pcfg(True)
        cfg["sequence_packing"]["microbatch_order"] = order
        cfg["sequence_packing"]["max_sequences_per_bin"] = 2
        w = PolicyWorker(cfg, model_cfg=TINY, seed=3)
        lens = [5, 30, 12, 40, 7, 22]
        plan = w._plan(lens, list(range(6)), 64)
        assert all(len(b) <= 2 for b in plan) and sorted(r for b in plan for r in b) == list(range(6))
        if order == "largest_first":
            tok = [sum(lens[r] for r in b) for b in plan]
            assert tok == sorted(tok, reverse=True)
        losses.append(w.train(make_batch(), ClippedPGLossFn({}), gbs=8)["loss"])
    assert abs(float(losses[0]) - float(losses[1])) < 1e-4
    with pytest.raises(ValueError, match="microbatch_order"):
        cfg = _pcfg(True)
        cfg["sequence_packing"]["microbatch_order"] = "smallest"
        PolicyWorker(cfg, model_cfg=TINY, seed=3)
