"""Context parallelism: load-balanced causal sequence sharding and attention
over the gathered keys / values.

Layout (the reference's, ``nemo_rl/distributed/model_utils.py:1234-1268``): every
sequence is padded to a multiple of ``2 * cp`` chunks; CP rank ``r`` holds chunks
``r`` and ``2cp - 1 - r``, so every rank carries the same causal-attention work.
A rank's packed stream is, per sequence, its two chunks back to back, with
their absolute positions.

Attention: the ranks' keys / values are gathered over the CP group (rank-major
order), re-ordered to the natural order of every sequence, and each local query
chunk attends to the prefix of its sequence up to its own last token (causal,
bottom-right aligned).  On CUDA this runs in the varlen flash-attention
kernels with per-segment key ranges (``csrc/attention.cu``); the torch
reference below is the CPU path and the test oracle.  The gather's backward
reduce-scatters the key / value gradients to their owners.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

__all__ = ["CPLayout", "cp_layout", "cp_attention", "gather_kv_cp", "attention_segments_ref", "CPKVExchange",
           "cp_attention_fused"]


@dataclass
class CPLayout:
    """Per micro-batch plan of one CP rank (all tensors on the model's device)."""
    cp: int
    rank: int
    local_index: torch.Tensor   # [T_local] index of each local token in the per-rank padded full stream
    positions: torch.Tensor     # [T_local] absolute positions (int32)
    valid: torch.Tensor         # [T_local] bool: real token (not chunk padding)
    # attention segments: one per local chunk
    q_start: torch.Tensor       # [S] first local row of the chunk
    q_len: torch.Tensor         # [S]
    k_start: torch.Tensor       # [S] first row of the chunk's sequence in the natural-order gathered K/V
    k_len: torch.Tensor         # [S] keys visible to the chunk (its sequence prefix through its last token)
    perm: torch.Tensor          # [T_full] natural-order row -> rank-major gathered row
    T_local: int
    T_full: int
    max_q: int
    max_k: int
    seq_of_local: torch.Tensor  # [T_local] which packed sequence each local token belongs to
    padded_len: list
    perm_inv_local: torch.Tensor = None  # [T_local] natural-order row of each local token
    pieces: dict = None                  # rank -> [(natural row, row in that rank's local stream, rows)]


def cp_layout(lengths: list[int], cp: int, rank: int, device, unit: int = 1) -> CPLayout:
    """Plan for sequences of ``lengths`` (already in packing order).  Every
    chunk length is a multiple of ``unit`` (so per-rank token counts stay
    aligned, e.g. for fused kernels)."""
    two = 2 * cp
    per_rank_tokens = 0
    padded = []
    for L in lengths:
        m = two * unit
        Lp = max(m, (int(L) + m - 1) // m * m)
        padded.append(Lp)
        per_rank_tokens += Lp // cp
    # natural full stream (per sequence, chunk order 0..2cp-1) and rank-major gathered stream
    loc_idx, pos, valid, seq_of = [], [], [], []
    q_start, q_len, k_start, k_len = [], [], [], []
    nat_to_gathered = []
    full_off = 0
    local_off = 0
    # offsets of each sequence inside every rank's local stream (identical on all ranks)
    seq_local_off = []
    o = 0
    for Lp in padded:
        seq_local_off.append(o)
        o += Lp // cp
    for s, (L, Lp) in enumerate(zip(lengths, padded)):
        c = Lp // two
        mine = (rank, two - 1 - rank)
        for j, ch in enumerate(mine):
            a = ch * c
            q_start.append(local_off + j * c)
            q_len.append(c)
            k_start.append(full_off)
            k_len.append(a + c)
            for t in range(c):
                p = a + t
                pos.append(p)
                valid.append(p < L)
                seq_of.append(s)
        local_off += 2 * c
        for ch in range(two):
            owner = ch if ch < cp else two - 1 - ch
            slot = 0 if ch < cp else 1
            base = owner * per_rank_tokens + seq_local_off[s] + slot * c
            nat_to_gathered.extend(range(base, base + c))
        full_off += Lp
    loc_idx = list(range(local_off))
    # contiguous pieces (one per sequence chunk) of every rank's local stream in natural order
    pieces = {r: [] for r in range(cp)}
    nat_local = []
    full_off2 = 0
    for s, Lp in enumerate(padded):
        c = Lp // two
        for ch in range(two):
            owner = ch if ch < cp else two - 1 - ch
            slot = 0 if ch < cp else 1
            pieces[owner].append((full_off2 + ch * c, seq_local_off[s] + slot * c, c))
        for ch in (rank, two - 1 - rank):
            nat_local.extend(range(full_off2 + ch * c, full_off2 + (ch + 1) * c))
        full_off2 += Lp
    dev = torch.device(device)
    i32 = dict(dtype=torch.int32, device=dev)
    return CPLayout(cp=cp, rank=rank, local_index=torch.tensor(loc_idx, dtype=torch.long, device=dev),
                    positions=torch.tensor(pos, **i32), valid=torch.tensor(valid, dtype=torch.bool, device=dev),
                    q_start=torch.tensor(q_start, **i32), q_len=torch.tensor(q_len, **i32),
                    k_start=torch.tensor(k_start, **i32), k_len=torch.tensor(k_len, **i32),
                    perm=torch.tensor(nat_to_gathered, dtype=torch.long, device=dev), T_local=local_off,
                    T_full=full_off, max_q=max(q_len) if q_len else 0, max_k=max(k_len) if k_len else 0,
                    seq_of_local=torch.tensor(seq_of, dtype=torch.long, device=dev), padded_len=padded,
                    perm_inv_local=torch.tensor(nat_local, dtype=torch.long, device=dev), pieces=pieces)


class _GatherCP(torch.autograd.Function):
    """All-gather of [T_local, ...] rows over the CP group (rank-major);
    backward: reduce-scatter."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        out = torch.empty((x.shape[0] * n,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        n = dist.get_world_size(ctx.group)
        out = torch.empty((g.shape[0] // n,) + tuple(g.shape[1:]), dtype=g.dtype, device=g.device)
        dist.reduce_scatter_tensor(out, g.contiguous(), group=ctx.group)
        return out, None


def gather_kv_cp(x: torch.Tensor, layout: CPLayout, group) -> torch.Tensor:
    """Local [T_local, nkv, hd] -> natural-order [T_full, nkv, hd]."""
    g = _GatherCP.apply(x, group)
    return g.index_select(0, layout.perm)


def attention_segments_ref(q, k, v, layout: CPLayout, scale: float) -> torch.Tensor:
    """fp32 torch reference: q [T_local, nq, hd], k/v natural order [T_full, nkv, hd]."""
    nq, nkv = q.shape[1], k.shape[1]
    G = nq // nkv
    out = torch.zeros_like(q)
    for s in range(layout.q_start.numel()):
        qs, ql = int(layout.q_start[s]), int(layout.q_len[s])
        ks, kl = int(layout.k_start[s]), int(layout.k_len[s])
        qq = q[qs:qs + ql].float()                                   # [ql, nq, hd]
        kk = k[ks:ks + kl].float().repeat_interleave(G, 1)           # [kl, nq, hd]
        vv = v[ks:ks + kl].float().repeat_interleave(G, 1)
        sc = torch.einsum("qhd,khd->hqk", qq, kk) * scale
        qpos = torch.arange(kl - ql, kl, device=q.device)
        mask = torch.arange(kl, device=q.device)[None, :] > qpos[:, None]
        sc = sc.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(sc, -1)
        out[qs:qs + ql] = torch.einsum("hqk,khd->qhd", p, vv).to(q.dtype)
    return out


def cp_attention(q, k_full, v_full, layout: CPLayout, scale: float) -> torch.Tensor:
    """Local query chunks against their sequence prefixes (see module docstring)."""
    if q.is_cuda:
        from rl_b200.ops.attention import flash_attn_segments

        return flash_attn_segments(q, k_full, v_full, layout.q_start, layout.q_len, layout.k_start, layout.k_len,
                                   layout.max_q, layout.max_k, scale)
    return attention_segments_ref(q, k_full, v_full, layout, scale)


class CPKVExchange:
    """Context-parallel K/V exchange overlapped with the attention kernel.

    Each call publishes this rank's local K and V rows into a symmetric slot
    (double-buffered by call parity), places its own chunks at their natural
    positions, fences the CP group (tiny NCCL all-reduce), and then a side
    stream pulls every peer's chunks with copy-engine transfers over NVLink
    straight into their natural positions, writing the peer's flag (stream
    memory op, no kernel) after each peer.  The segment-attention kernel starts
    at once and waits per key block only for the chunk's owner: local chunks
    first, remote ones as they land."""

    def __init__(self, group, max_local_rows: int, row_elems: int):
        from rl_b200.parallel.symm import SymmetricBuffer

        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.max_rows = int(max_local_rows)
        self.E = int(row_elems)  # nkv * hd
        # per slot: K rows then V rows
        self.slot_elems = 2 * self.max_rows * self.E
        self.slots = SymmetricBuffer(2 * self.slot_elems * 2, group)
        self.flags = torch.zeros(max(self.n, 4), dtype=torch.int32, device="cuda")
        self.side = torch.cuda.Stream()
        self.epoch = 0
        self._fence = torch.zeros(1, device="cuda")

    def __call__(self, k: torch.Tensor, v: torch.Tensor, lay: CPLayout):
        from rl_b200.ops._ext import ext

        T = k.shape[0]
        if T > self.max_rows or k[0].numel() != self.E:
            raise ValueError("K/V exchange sized for fewer rows")
        self.epoch += 1
        par = self.epoch & 1
        e = ext()
        main = torch.cuda.current_stream()
        base = par * self.slot_elems
        mine_k = self.slots.local_view(torch.bfloat16, T * self.E, offset_bytes=base * 2).view(T, -1)
        mine_v = self.slots.local_view(torch.bfloat16, T * self.E,
                                       offset_bytes=(base + self.max_rows * self.E) * 2).view(T, -1)
        mine_k.copy_(k.reshape(T, -1))
        mine_v.copy_(v.reshape(T, -1))
        kf = torch.empty((lay.T_full,) + tuple(k.shape[1:]), dtype=k.dtype, device=k.device)
        vf = torch.empty_like(kf)
        own = lay.perm_inv_local  # natural rows of this rank's local tokens
        kf.index_copy_(0, own, k)
        vf.index_copy_(0, own, v)
        e.stream_write_u32(self.flags.data_ptr() + 4 * self.me, self.epoch)
        dist.all_reduce(self._fence, group=self.group)  # every rank published (a kernel: before the attention)
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            for j in range(1, self.n):
                src = (self.me + j) % self.n
                pk = self.slots.ptrs[src] + base * 2
                pv = self.slots.ptrs[src] + (base + self.max_rows * self.E) * 2
                for (nat0, loc0, rows) in lay.pieces[src]:
                    _copy_rows(kf, nat0, pk, loc0, rows, self.E)
                    _copy_rows(vf, nat0, pv, loc0, rows, self.E)
                e.stream_write_u32(self.flags.data_ptr() + 4 * src, self.epoch)
        kf.record_stream(self.side)
        vf.record_stream(self.side)
        return kf, vf

    def close(self) -> None:
        self.slots.close()


def _copy_rows(dst: torch.Tensor, dst_row: int, src_ptr: int, src_row: int, rows: int, E: int) -> None:
    from rl_b200.ops._ext import ext

    src = ext().symm_view(src_ptr + src_row * E * 2, rows * E, 15, dst.device.index)
    dst.view(dst.shape[0], -1)[dst_row:dst_row + rows].view(-1).copy_(src, non_blocking=True)


class _CPAttentionFused(torch.autograd.Function):
    """Segment attention whose K/V gather overlaps the kernel (``CPKVExchange``);
    backward: segment-attention gradients in the natural layout, moved to the
    rank-major layout and reduce-scattered to the owners."""

    @staticmethod
    def forward(ctx, q, k, v, lay, exch, scale):
        from rl_b200.ops._ext import ext

        kf, vf = exch(k, v, lay)
        seg = torch.stack([lay.q_start, lay.q_len, lay.k_start, lay.k_len], 1).to(torch.int32).contiguous()
        from rl_b200.ops.attention import fa_seg_forward

        o, lse = fa_seg_forward(q.contiguous(), kf, vf, seg, int(lay.max_q), float(scale), exch.flags, exch.epoch,
                                exch.n)
        torch.cuda.current_stream().wait_stream(exch.side)
        ctx.save_for_backward(q, kf, vf, o, lse, seg)
        ctx.lay, ctx.scale, ctx.group = lay, scale, exch.group
        return o

    @staticmethod
    def backward(ctx, do):
        from rl_b200.ops._ext import ext

        q, kf, vf, o, lse, seg = ctx.saved_tensors
        lay = ctx.lay
        from rl_b200.ops.attention import fa_seg_backward

        dq, dk_n, dv_n = fa_seg_backward(do, q, kf, vf, o, lse, seg, int(lay.max_k), float(ctx.scale))
        n = dist.get_world_size(ctx.group)
        outs = []
        for g in (dk_n, dv_n):
            rm = torch.empty_like(g)
            rm.index_copy_(0, lay.perm, g)  # natural row i lives at rank-major row perm[i]
            loc = torch.empty((g.shape[0] // n,) + tuple(g.shape[1:]), dtype=g.dtype, device=g.device)
            dist.reduce_scatter_tensor(loc, rm, group=ctx.group)
            outs.append(loc)
        return dq, outs[0], outs[1], None, None, None


def cp_attention_fused(q, k, v, lay: CPLayout, exch: CPKVExchange, scale: float) -> torch.Tensor:
    return _CPAttentionFused.apply(q, k, v, lay, exch, scale)
