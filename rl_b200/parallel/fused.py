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

__all__ = ["GemmReduceScatter", "row_parallel_rs", "AllGatherGemm", "column_parallel_ag", "DecodeAllReduceNorm"]


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


class _ColumnParallelAG(torch.autograd.Function):
    """y = AG(x_shard) @ w^T with the all-gather overlapped inside the GEMM;
    backward: input gradient GEMM then NCCL reduce-scatter to the shard, weight
    gradient into main_grad from the gathered input."""

    @staticmethod
    def forward(ctx, x, w, op):
        y, gathered = op(x, w)
        ctx.save_for_backward(gathered, w)
        ctx.op = op
        return y

    @staticmethod
    def backward(ctx, dy):
        from rl_b200.ops import gemm as _gemm

        g, w = ctx.saved_tensors
        op = ctx.op
        dy = dy.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            full = _gemm.mm_nn(dy, w)
            dx = torch.empty((full.shape[0] // op.n, full.shape[1]), dtype=full.dtype, device=full.device)
            dist.reduce_scatter_tensor(dx, full, group=op.group)
        dw = None
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                _gemm.mm_tn_accumulate(dy, g, main)
            else:
                dw = _gemm.mm_tn(dy, g).to(w.dtype)
        return dx, dw, None


def column_parallel_ag(x: torch.Tensor, w: torch.Tensor, op: "AllGatherGemm") -> torch.Tensor:
    return _ColumnParallelAG.apply(x, w, op)


class AllGatherGemm:
    """``y = all_gather_rows(x_shard) @ w^T`` over the ranks of ``group`` (one
    node): the column-parallel linear of tensor parallelism with sequence
    parallelism, in which the gather overlaps the GEMM.

    Each call publishes this rank's shard into a symmetric slot (double-buffered
    by epoch parity) and fences the group (tiny NCCL all-reduce: every rank has
    published); then a side stream pulls every peer's shard with copy-engine
    transfers over NVLink into the local gathered buffer and, after each, writes
    that shard's flag with a stream memory op (no kernel, so the side stream
    never waits for an SM the GEMM holds).  The tcgen05 GEMM
    (``csrc/gemm_tcgen05.cu``, ``EPI=2``) starts on the own rows at once and waits
    on a remote shard's flag only when it reaches that shard's tiles.  No SM
    work is spent on the transfer and every remote byte crosses NVLink once.
    A slot is rewritten two calls later, after the next call's fence, which
    every peer enters only after its transfers of this call completed, so a
    slot is never overwritten while a peer still reads it."""

    BM = 128

    def __init__(self, group, max_rows: int, k: int):
        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.K = int(k)
        unit = self.BM * self.n
        self.max_rows = (int(max_rows) + unit - 1) // unit * unit
        self.ms_max = self.max_rows // self.n
        self.slots = SymmetricBuffer(2 * self.ms_max * self.K * 2, group)
        self.flags = torch.zeros(max(self.n, 4), dtype=torch.int32, device="cuda")
        self.side = torch.cuda.Stream()
        self.epoch = 0
        self._fence_buf = torch.zeros(1, device="cuda")

    def __call__(self, x: torch.Tensor, w: torch.Tensor):
        ms = x.shape[0]
        if ms % self.BM or ms > self.ms_max or x.shape[1] != self.K:
            raise ValueError(f"shard rows {ms} must be a multiple of {self.BM} and <= {self.ms_max}")
        x = x.contiguous()
        M = ms * self.n
        self.epoch += 1
        par = self.epoch & 1
        e = ext()
        main = torch.cuda.current_stream()
        slot_bytes = self.ms_max * self.K * 2
        mine = self.slots.local_view(torch.bfloat16, ms * self.K, offset_bytes=par * slot_bytes).view(ms, self.K)
        mine.copy_(x)
        gathered = torch.empty((M, self.K), dtype=x.dtype, device=x.device)
        gathered[self.me * ms:(self.me + 1) * ms].copy_(x)
        e.stream_write_u32(self.flags.data_ptr() + 4 * self.me, self.epoch)
        # every rank has published `mine` (and, a call earlier, finished reading the
        # slot this publish reused).  The fence is a kernel, so it runs here, before
        # the GEMM, never behind it: the side stream below needs no SM at all
        dist.all_reduce(self._fence_buf, group=self.group)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            for j in range(1, self.n):
                src = (self.me + j) % self.n
                peer = self.slots.ptrs[src] + par * slot_bytes
                _copy_from_ptr(gathered[src * ms:(src + 1) * ms], peer)
                e.stream_write_u32(self.flags.data_ptr() + 4 * src, self.epoch)
        gathered.record_stream(self.side)
        y = e.gemm_ag(gathered, w.contiguous(), self.flags, self.n, self.me, self.epoch)
        # later work of this stream (the next publish) runs after the transfers
        main.wait_stream(self.side)
        return y, gathered

    def close(self) -> None:
        self.slots.close()


def _copy_from_ptr(dst: torch.Tensor, src_ptr: int) -> None:
    """Copy-engine transfer of ``dst.numel()`` bf16 elements from a (peer) device
    address into ``dst`` on the current stream."""
    src = ext().symm_view(src_ptr, dst.numel(), 15, dst.device.index)
    dst.view(-1).copy_(src, non_blocking=True)


class DecodeAllReduceNorm:
    """Decode-step TP all-reduce fused with the residual add and RMSNorm
    (``csrc/decode_ar.cu``): ``h = RMSNorm(resid + sum_r partial_r) * w`` with
    ``resid`` updated in place, over symmetric slots and per-row flags of the TP
    group.  The epoch lives in a device counter, so the op replays in CUDA graphs;
    it must be created (collective) outside graph capture."""

    def __init__(self, group, cap: int, H: int):
        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.cap, self.H = int(cap), int(H)
        self.slots = SymmetricBuffer(2 * self.cap * self.H * 2, group)
        self.flags = SymmetricBuffer(self.n * self.cap * 4, group)
        self.ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.done = torch.zeros(1, dtype=torch.int32, device="cuda")

    def __call__(self, partial: torch.Tensor, resid: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
        return ext().ar_add_rmsnorm(partial.contiguous(), resid, w, float(eps), self.slots.ptrs, self.flags.ptrs,
                                    self.me, self.cap, self.ctr, self.done)

    def close(self) -> None:
        self.slots.close()
        self.flags.close()
