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

__all__ = ["CPLayout", "cp_layout", "cp_attention", "gather_kv_cp", "attention_segments_ref"]


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
    dev = torch.device(device)
    i32 = dict(dtype=torch.int32, device=dev)
    return CPLayout(cp=cp, rank=rank, local_index=torch.tensor(loc_idx, dtype=torch.long, device=dev),
                    positions=torch.tensor(pos, **i32), valid=torch.tensor(valid, dtype=torch.bool, device=dev),
                    q_start=torch.tensor(q_start, **i32), q_len=torch.tensor(q_len, **i32),
                    k_start=torch.tensor(k_start, **i32), k_len=torch.tensor(k_len, **i32),
                    perm=torch.tensor(nat_to_gathered, dtype=torch.long, device=dev), T_local=local_off,
                    T_full=full_off, max_q=max(q_len) if q_len else 0, max_k=max(k_len) if k_len else 0,
                    seq_of_local=torch.tensor(seq_of, dtype=torch.long, device=dev), padded_len=padded)


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
