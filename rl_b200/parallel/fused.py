"""Fused compute + collective ops over NVLink peer memory.

``GemmReduceScatter``: ``out_r = (sum_ranks A_rank @ W_rank^T)[rows of rank r]`` -
the row-parallel linear of tensor parallelism with sequence parallelism - as ONE
tcgen05 kernel per rank (``csrc/gemm_tcgen05.cu``, epilogue ``EPI=1``): tiles
destined to a peer are stored straight into the peer's receive buffer over
NVLink as they finish (so the transfer overlaps the remaining MMA work), own
tiles wait for the peers' partials and reduce them in the epilogue.  The NCCL
baseline it replaces is ``GEMM`` then ``reduce_scatter_tensor``.

The op keeps symmetric receive / flag / ack buffers sized for ``max_rows`` rows
and an epoch counter that advances identically on every rank (all ranks of the
group must call it in the same order).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from rl_b200.ops._ext import ext
from rl_b200.parallel.symm import SymmetricBuffer

__all__ = ["GemmReduceScatter", "row_parallel_rs"]


class _RowParallelRS(torch.autograd.Function):
    """y_shard = RS(x @ w^T) fused forward; backward gathers dy over TP and runs
    the input / weight gradient GEMMs (weight gradient straight into main_grad)."""

    @staticmethod
    def forward(ctx, x, w, op):
        ctx.save_for_backward(x, w)
        ctx.op = op
        return op(x, w)

    @staticmethod
    def backward(ctx, dy):
        from rl_b200.ops import gemm as _gemm

        x, w = ctx.saved_tensors
        op = ctx.op
        full = torch.empty((dy.shape[0] * op.n, dy.shape[1]), dtype=dy.dtype, device=dy.device)
        dist.all_gather_into_tensor(full, dy.contiguous(), group=op.group)
        dx = _gemm.mm_nn(full, w) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                _gemm.mm_tn_accumulate(full, x, main)
            else:
                dw = _gemm.mm_tn(full, x).to(w.dtype)
        return dx, dw, None


def row_parallel_rs(x: torch.Tensor, w: torch.Tensor, op: "GemmReduceScatter") -> torch.Tensor:
    return _RowParallelRS.apply(x, w, op)


class GemmReduceScatter:
    BM = 128

    def __init__(self, group, max_rows: int, n_cols: int):
        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.N = int(n_cols)
        unit = self.BM * self.n
        self.max_rows = (int(max_rows) + unit - 1) // unit * unit
        ms = self.max_rows // self.n
        bn = 256 if self.N >= 256 else 128
        self.tiles_per_shard = (ms // self.BM) * ((self.N + bn - 1) // bn)
        self.recv = SymmetricBuffer(2 * self.n * ms * self.N * 2, group)
        self.flags = SymmetricBuffer(2 * self.n * self.tiles_per_shard * 4, group)
        self.acks = SymmetricBuffer((2 * self.n + 2) * 4, group)  # per-parity ack words + launch counters
        self.epoch = 0
        self._shape_ms = None

    def __call__(self, a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        M = a.shape[0]
        if M % (self.BM * self.n) or M > self.max_rows:
            raise ValueError(f"rows {M} must be a multiple of {self.BM * self.n} and <= {self.max_rows}")
        ms = M // self.n
        if self._shape_ms is not None and self._shape_ms != ms:
            # the per-tile flag indexing depends on the shard height: keep epochs
            # monotone (flags / acks compare against the epoch, never reset)
            pass
        self._shape_ms = ms
        out = torch.empty(ms, self.N, dtype=a.dtype, device=a.device)
        self.epoch += 1
        ext().gemm_rs(a.contiguous(), w.contiguous(), out, self.recv.ptrs, self.flags.ptrs, self.acks.ptrs, self.me,
                      self.epoch)
        return out

    def close(self) -> None:
        for b in (self.recv, self.flags, self.acks):
            b.close()
