"""Autograd-aware collectives for tensor / sequence / expert parallelism.

The four tensor-parallel region markers of Megatron-style TP (identity/all-reduce
pairs and their sequence-parallel all-gather/reduce-scatter variants), plus an
autograd all-to-all for expert dispatch.  These are the NCCL baseline paths;
the fused compute+collective kernels in ``rl_b200.parallel.fused`` replace the
GEMM-adjacent ones on NVLink.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

__all__ = [
    "copy_to_tp", "reduce_from_tp", "gather_from_sp", "reduce_scatter_to_sp", "scatter_to_sp",
    "all_to_all_autograd", "all_reduce_sum",
]


def _ws(group) -> int:
    return 1 if group is None else dist.get_world_size(group)


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherFromSP(torch.autograd.Function):
    """Forward: all-gather along dim 0; backward: reduce-scatter."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = _ws(group)
        out = torch.empty((x.shape[0] * n, *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        n = _ws(ctx.group)
        out = torch.empty((g.shape[0] // n, *g.shape[1:]), dtype=g.dtype, device=g.device)
        dist.reduce_scatter_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


class _ReduceScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = _ws(group)
        out = torch.empty((x.shape[0] // n, *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        n = _ws(ctx.group)
        out = torch.empty((g.shape[0] * n, *g.shape[1:]), dtype=g.dtype, device=g.device)
        dist.all_gather_into_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


class _ScatterToSP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = _ws(group)
        r = dist.get_rank(group)
        chunk = x.shape[0] // n
        return x[r * chunk:(r + 1) * chunk].contiguous()

    @staticmethod
    def backward(ctx, g):
        n = _ws(ctx.group)
        out = torch.empty((g.shape[0] * n, *g.shape[1:]), dtype=g.dtype, device=g.device)
        dist.all_gather_into_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


def copy_to_tp(x, group):
    return x if _ws(group) == 1 else _CopyToTP.apply(x, group)


def reduce_from_tp(x, group):
    return x if _ws(group) == 1 else _ReduceFromTP.apply(x, group)


def gather_from_sp(x, group):
    return x if _ws(group) == 1 else _GatherFromSP.apply(x, group)


def reduce_scatter_to_sp(x, group):
    return x if _ws(group) == 1 else _ReduceScatterToSP.apply(x, group)


def scatter_to_sp(x, group):
    return x if _ws(group) == 1 else _ScatterToSP.apply(x, group)


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_splits, recv_splits, group):
        ctx.group = group
        ctx.send_splits, ctx.recv_splits = send_splits, recv_splits
        out = torch.empty((sum(recv_splits), *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = torch.empty((sum(ctx.send_splits), *g.shape[1:]), dtype=g.dtype, device=g.device)
        dist.all_to_all_single(out, g.contiguous(), ctx.send_splits, ctx.recv_splits, group=ctx.group)
        return out, None, None, None


def all_to_all_autograd(x: torch.Tensor, send_splits: list[int], recv_splits: list[int], group) -> torch.Tensor:
    return _AllToAll.apply(x, send_splits, recv_splits, group)


def all_reduce_sum(x: torch.Tensor, group=None) -> torch.Tensor:
    if dist.is_available() and dist.is_initialized() and _ws(group) > 1:
        dist.all_reduce(x, group=group)
    return x
