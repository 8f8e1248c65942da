"""Process-group layout for TP / CP / EP / DP / PP on one node (or several).

One process per GPU.  Rank order (fastest-varying first): TP, CP, DP, PP - so
tensor-parallel peers are adjacent GPUs (same NVSwitch domain, lowest latency)
and each DP replica holds a contiguous block of ranks.  EP reuses the DP x CP x
TP ranks of a pipeline stage in the same fastest-first order (expert-parallel
groups are formed over ``ep_size`` consecutive ranks of the non-TP ranks,
matching MCore's default where EP groups are carved out of DP).

Reference: ``nemo_rl/models/megatron/setup.py:534`` (``setup_distributed``) and
``:1299`` (``_apply_parallelism_config``), ``nemo_rl/distributed/named_sharding.py:31``.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

__all__ = ["ParallelState", "init_distributed", "get_parallel_state", "set_parallel_state", "single_process_state"]


@dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    local_rank: int = 0
    tp_size: int = 1
    cp_size: int = 1
    ep_size: int = 1
    pp_size: int = 1
    dp_size: int = 1
    tp_rank: int = 0
    cp_rank: int = 0
    ep_rank: int = 0
    pp_rank: int = 0
    dp_rank: int = 0
    tp_group: Optional[object] = None
    cp_group: Optional[object] = None
    ep_group: Optional[object] = None
    pp_group: Optional[object] = None
    dp_group: Optional[object] = None
    dp_cp_group: Optional[object] = None
    mp_group: Optional[object] = None  # TP x CP x PP (all ranks of one model replica)
    edp_group: Optional[object] = None  # expert-data-parallel: ranks holding the same experts
    edp_ranks: list = field(default_factory=lambda: [0])
    tp_ranks: list = field(default_factory=lambda: [0])
    dp_ranks: list = field(default_factory=lambda: [0])
    ep_ranks: list = field(default_factory=lambda: [0])
    cp_ranks: list = field(default_factory=lambda: [0])
    pp_ranks: list = field(default_factory=lambda: [0])
    backend: str = "gloo"
    device: torch.device = field(default_factory=lambda: torch.device("cpu"))

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


_STATE: Optional[ParallelState] = None


def single_process_state(device: Optional[torch.device] = None) -> ParallelState:
    return ParallelState(device=device or torch.device("cpu"))


def set_parallel_state(st: ParallelState) -> None:
    global _STATE
    _STATE = st


def get_parallel_state() -> ParallelState:
    global _STATE
    if _STATE is None:
        _STATE = single_process_state()
    return _STATE


def rank_coords(rank: int, tp: int, cp: int, dp: int, pp: int) -> tuple[int, int, int, int]:
    t = rank % tp
    c = (rank // tp) % cp
    d = (rank // (tp * cp)) % dp
    p = rank // (tp * cp * dp)
    return t, c, d, p


def init_distributed(tp: int = 1, cp: int = 1, ep: int = 1, pp: int = 1, backend: Optional[str] = None,
                     timeout_s: float = 600.0) -> ParallelState:
    """Initialise ``torch.distributed`` from the torchrun environment (or a single
    process when ``WORLD_SIZE`` is unset) and build every sub-group."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available()
    if backend is None:
        backend = "nccl" if use_cuda else "gloo"
    device = torch.device("cuda", local_rank) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {}
        if backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(backend=backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    if world % (tp * cp * pp) != 0:
        raise ValueError(f"world size {world} not divisible by tp*cp*pp = {tp * cp * pp}")
    dp = world // (tp * cp * pp)
    if (dp * cp * tp) % (ep * tp) != 0 and ep > 1:
        raise ValueError(f"expert parallel size {ep} must divide dp*cp = {dp * cp}")
    st = ParallelState(world_size=world, rank=rank, local_rank=local_rank, tp_size=tp, cp_size=cp, ep_size=ep,
                       pp_size=pp, dp_size=dp, backend=backend, device=device)
    st.tp_rank, st.cp_rank, st.dp_rank, st.pp_rank = rank_coords(rank, tp, cp, dp, pp)
    if world == 1:
        set_parallel_state(st)
        return st

    def make(groups: list[list[int]], attr: str, ranks_attr: Optional[str] = None):
        for g in groups:
            # the job's timeout, not the library default: ranks that wait on a lost
            # peer in a sub-group collective end with an error instead of hanging
            pg = dist.new_group(g, backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
            if rank in g:
                setattr(st, attr, pg)
                if ranks_attr:
                    setattr(st, ranks_attr, g)

    all_ranks = list(range(world))
    coords = {r: rank_coords(r, tp, cp, dp, pp) for r in all_ranks}
    # TP groups: vary t
    make([[r for r in all_ranks if coords[r][1:] == key] for key in sorted({c[1:] for c in coords.values()})],
         "tp_group", "tp_ranks")
    # CP groups: vary c, fixed (t, d, p)
    make([[r for r in all_ranks if (coords[r][0], coords[r][2], coords[r][3]) == key]
          for key in sorted({(c[0], c[2], c[3]) for c in coords.values()})], "cp_group", "cp_ranks")
    # DP groups: vary d, fixed (t, c, p)
    make([[r for r in all_ranks if (coords[r][0], coords[r][1], coords[r][3]) == key]
          for key in sorted({(c[0], c[1], c[3]) for c in coords.values()})], "dp_group", "dp_ranks")
    # DP x CP groups (gradient reduction domain): fixed (t, p)
    make([[r for r in all_ranks if (coords[r][0], coords[r][3]) == key]
          for key in sorted({(c[0], c[3]) for c in coords.values()})], "dp_cp_group")
    # PP groups: vary p
    make([[r for r in all_ranks if coords[r][:3] == key] for key in sorted({c[:3] for c in coords.values()})],
         "pp_group", "pp_ranks")
    # Model-parallel groups (one replica): fixed d
    make([[r for r in all_ranks if coords[r][2] == d] for d in range(dp)], "mp_group")
    # EP groups: within a pipeline stage and TP rank, consecutive blocks of ep ranks
    # among the (c, d) coordinates.
    ep_groups = []
    for p in range(pp):
        for t in range(tp):
            members = [r for r in all_ranks if coords[r][3] == p and coords[r][0] == t]
            for i in range(0, len(members), ep):
                ep_groups.append(members[i:i + ep])
    make(ep_groups, "ep_group", "ep_ranks")
    st.ep_rank = st.ep_ranks.index(rank) if rank in st.ep_ranks else 0
    # Expert-data-parallel groups: ranks holding the SAME experts (same position in
    # their EP group) within a pipeline stage / TP rank; expert gradients are
    # reduced over these only.
    edp_groups = []
    for p in range(pp):
        for t in range(tp):
            blocks = [g for g in ep_groups if coords[g[0]][3] == p and coords[g[0]][0] == t]
            for e in range(ep):
                edp_groups.append([blk[e] for blk in blocks if e < len(blk)])
    make(edp_groups, "edp_group", "edp_ranks")
    set_parallel_state(st)
    return st
