"""NamedSharding: the reference's layout API, and the layout of this
framework's process grid agreeing with every rank's coordinates (CPU)."""

import pytest

from rl_b200.distributed.named_sharding import NamedSharding, from_parallel_state


def test_named_sharding_api():
    s = NamedSharding([[[0, 1, 2, 3], [4, 5, 6, 7]]], ["dp", "pp", "tp"])
    assert s.shape == {"dp": 1, "pp": 2, "tp": 4} and s.size == 8 and s.ndim == 3
    sub = s.get_ranks(dp=0, pp=1)
    assert isinstance(sub, NamedSharding) and sub.names == ["tp"] and sub.layout.tolist() == [4, 5, 6, 7]
    assert s.get_ranks(dp=0, pp=1, tp=2) == 6
    assert s.get_ranks_by_coord(tp=1) == [1, 5] and s.get_ranks_by_coord(pp=5) == []
    assert s.get_worker_coords(6) == {"dp": 0, "pp": 1, "tp": 2}
    assert s.get_axis_size("tp") == 4 and s.get_axis_index("pp") == 1
    assert NamedSharding.is_axis_zero({"dp": 0, "pp": 1}, ["dp", "cp"])
    assert s == NamedSharding([[[0, 1, 2, 3], [4, 5, 6, 7]]], ["dp", "pp", "tp"])
    with pytest.raises(ValueError):
        NamedSharding([[0, 0]], ["a", "b"])  # duplicate rank
    with pytest.raises(ValueError):
        NamedSharding([0, 1], ["a", "b"])  # dimension mismatch
    with pytest.raises(IndexError):
        s.get_ranks(pp=2)
    with pytest.raises(ValueError):
        s.get_axis_size("ep")


def test_layout_of_the_process_grid():
    from rl_b200.parallel.state import ParallelState, rank_coords

    tp, cp, dp, pp = 2, 2, 3, 2
    ps = ParallelState(world_size=tp * cp * dp * pp, tp_size=tp, cp_size=cp, dp_size=dp, pp_size=pp)
    s = from_parallel_state(ps)
    assert s.shape == {"pipeline_parallel": 2, "data_parallel": 3, "context_parallel": 2, "tensor_parallel": 2}
    for r in range(ps.world_size):
        t, c, d, p = rank_coords(r, tp, cp, dp, pp)
        assert s.get_worker_coords(r) == {"pipeline_parallel": p, "data_parallel": d, "context_parallel": c,
                                          "tensor_parallel": t}
    # the TP group of rank 5 = all ranks sharing its other coordinates
    c5 = s.get_worker_coords(5)
    grp = s.get_ranks_by_coord(**{k: v for k, v in c5.items() if k != "tensor_parallel"})
    assert 5 in grp and len(grp) == tp
