"""Attention ops: packed variable-length causal GQA attention (training and
prefill), paged-KV decode attention and KV-cache writes (rollout).

Reference counterparts: training attention is TE ``DotProductAttention`` over
packed THD sequences (native component N5, ``nemo_rl/models/megatron/data.py:1673``
builds the ``cu_seqlens``); rollout attention is vLLM / MCore paged attention
with ``block_size_tokens: 256`` (N15, ``examples/configs/grpo_math_1B.yaml:345``).

Layouts
-------
* packed: ``q [T, nq, hd]``, ``k, v [T, nkv, hd]`` (may be strided views of the
  QKV projection), ``cu_seqlens [B+1] int32``; output ``[T, nq, hd]`` and the
  per-row log-sum-exp ``lse [nq, T] fp32`` kept for the backward pass.
* paged cache: ``k_cache, v_cache [num_blocks, block_size, nkv, hd]``,
  ``block_tables [B, max_blocks] int32``, ``seq_lens [B] int32``;
  ``slot_mapping [T] int64`` = block * block_size + offset for writes.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch

from rl_b200.ops._ext import ext, use_native

__all__ = [
    "flash_attn_varlen",
    "flash_attn_varlen_ref",
    "paged_decode_attention",
    "paged_decode_attention_ref",
    "write_kv_cache",
    "write_kv_cache_ref",
]


def flash_attn_varlen_ref(q, k, v, cu_seqlens, scale: Optional[float] = None, causal: bool = True):
    """fp32 oracle: loop over packed sequences, explicit softmax."""
    T, nq, hd = q.shape
    nkv = k.shape[1]
    g = nq // nkv
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    out = torch.empty(T, nq, hd, dtype=torch.float32, device=q.device)
    lse = torch.empty(nq, T, dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        if e <= s:
            continue
        qb = q[s:e].float().transpose(0, 1)                                  # [nq, L, hd]
        kb = k[s:e].float().transpose(0, 1).repeat_interleave(g, dim=0)      # [nq, L, hd]
        vb = v[s:e].float().transpose(0, 1).repeat_interleave(g, dim=0)
        sc = torch.matmul(qb, kb.transpose(-1, -2)) * scale
        if causal:
            L = e - s
            m = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
            sc = sc.masked_fill(m, float("-inf"))
        lse[:, s:e] = torch.logsumexp(sc, -1)
        out[s:e] = torch.matmul(torch.softmax(sc, -1), vb).transpose(0, 1)
    return out.to(q.dtype), lse


# RL_B200_ATTN_TC=0 keeps the forward on the mma.sync kernel (A/B timing)
_ATTN_TC = os.environ.get("RL_B200_ATTN_TC", "1") == "1"
# RL_B200_ATTN_TC_BWD=0 keeps the backward on the mma.sync kernel (A/B timing)
_TC_BWD = os.environ.get("RL_B200_ATTN_TC_BWD", "1") == "1"


def _tc_ok(*xs) -> bool:
    """The tcgen05 forward (``csrc/attention_sm100.cu``) takes head dim 128 bf16 views
    with contiguous heads and 16-byte aligned token rows (TMA tensor maps)."""
    return _ATTN_TC and all(x.dim() == 3 and x.shape[-1] == 128 and x.dtype == torch.bfloat16 and x.stride(2) == 1
                            and x.stride(1) == 128 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0 for x in xs)


def fa_forward(q, k, v, cu_seqlens, max_seqlen: int, scale: float, causal: bool):
    """Native varlen forward: (out, lse) from the tcgen05 kernel when it applies."""
    if os.environ.get("RLB_PROBE_ATTN_FP32") == "1":  # numerics probe only: fp32 attention
        o, lse = flash_attn_varlen_ref(q.float(), k.float(), v.float(), cu_seqlens, scale, causal)
        return o.to(q.dtype), lse
    if _tc_ok(q, k, v):
        return ext().flash_attn_fwd_tc(q, k, v, cu_seqlens, int(max_seqlen), float(scale), bool(causal))
    return ext().flash_attn_fwd(q, k, v, cu_seqlens, int(max_seqlen), float(scale), bool(causal))


def fa_seg_forward(q, k, v, seg, max_q: int, scale: float, cp_flags=None, cp_epoch: int = 0, cp_size: int = 0):
    """Native segment forward (context parallelism), tcgen05 when it applies."""
    if _tc_ok(q, k, v):
        return ext().flash_attn_seg_fwd_tc(q, k, v, seg, int(max_q), float(scale), cp_flags, int(cp_epoch),
                                           int(cp_size))
    return ext().flash_attn_seg_fwd(q, k, v, seg, int(max_q), float(scale), cp_flags, int(cp_epoch), int(cp_size))


def fa_backward(do, q, k, v, o, lse, cu_seqlens, max_seqlen: int, scale: float, causal: bool):
    """Native varlen backward: (dq, dk, dv), tcgen05 kernel when it applies."""
    do = do.contiguous()
    if _TC_BWD and _tc_ok(q, k, v, do) and o.is_contiguous():
        return ext().flash_attn_bwd_tc(do, q, k, v, o, lse, cu_seqlens, int(max_seqlen), float(scale), bool(causal))
    return ext().flash_attn_bwd(do, q, k, v, o, lse, cu_seqlens, int(max_seqlen), float(scale), bool(causal))


def fa_seg_backward(do, q, k, v, o, lse, seg, max_k: int, scale: float):
    """Native segment backward (context parallelism), tcgen05 when it applies."""
    do = do.contiguous()
    if _TC_BWD and _tc_ok(q, k, v, do) and o.is_contiguous():
        return ext().flash_attn_seg_bwd_tc(do, q, k, v, o, lse, seg, int(max_k), float(scale))
    return ext().flash_attn_seg_bwd(do, q, k, v, o, lse, seg, int(max_k), float(scale))


class _FlashAttnVarlen(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_seqlen, scale, causal):
        o, lse = fa_forward(q, k, v, cu_seqlens, int(max_seqlen), float(scale), bool(causal))
        ctx.save_for_backward(q, k, v, o, lse, cu_seqlens)
        ctx.meta = (int(max_seqlen), float(scale), bool(causal))
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, cu = ctx.saved_tensors
        max_seqlen, scale, causal = ctx.meta
        dq, dk, dv = fa_backward(do, q, k, v, o, lse, cu, max_seqlen, scale, causal)
        return dq, dk, dv, None, None, None, None


def flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen: int, scale: Optional[float] = None, causal: bool = True):
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if use_native(q):
        return _FlashAttnVarlen.apply(q, k, v, cu_seqlens, max_seqlen, scale, causal)
    return flash_attn_varlen_ref(q, k, v, cu_seqlens, scale, causal)[0]


class _FlashAttnSegments(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seg, max_q, max_k, scale):
        o, lse = fa_seg_forward(q, k, v, seg, int(max_q), float(scale))
        ctx.save_for_backward(q, k, v, o, lse, seg)
        ctx.meta = (int(max_k), float(scale))
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, seg = ctx.saved_tensors
        max_k, scale = ctx.meta
        dq, dk, dv = fa_seg_backward(do, q, k, v, o, lse, seg, max_k, scale)
        return dq, dk, dv, None, None, None, None


def flash_attn_segments(q, k, v, q_start, q_len, k_start, k_len, max_q: int, max_k: int, scale: float):
    """Segment ``s`` attends queries ``[q_start[s], +q_len[s])`` to keys
    ``[k_start[s], +k_len[s])``, causal with the last query aligned to the last
    key (context-parallel chunks against their sequence prefixes; segments may
    share keys).  Native kernels: the varlen flash-attention kernels of
    ``csrc/attention.cu`` with per-segment ranges."""
    seg = torch.stack([q_start, q_len, k_start, k_len], 1).to(torch.int32).contiguous()
    return _FlashAttnSegments.apply(q.contiguous(), k.contiguous(), v.contiguous(), seg, max_q, max_k, scale)


def flash_attn_varlen_fwd(q, k, v, cu_seqlens, max_seqlen: int, scale: Optional[float] = None,
                          causal: bool = True):
    """Forward only (prefill): returns (out, lse)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if use_native(q):
        return fa_forward(q, k, v, cu_seqlens, int(max_seqlen), float(scale), bool(causal))
    return flash_attn_varlen_ref(q, k, v, cu_seqlens, scale, causal)


def write_kv_cache_ref(k, v, k_cache, v_cache, slot_mapping, k_scale: float = 1.0, v_scale: float = 1.0):
    nb, bs = k_cache.shape[:2]
    kc = k_cache.view(nb * bs, *k_cache.shape[2:])
    vc = v_cache.view(nb * bs, *v_cache.shape[2:])
    if kc.dtype == torch.float8_e4m3fn:
        k, v = (k.float() / k_scale).clamp(-448, 448), (v.float() / v_scale).clamp(-448, 448)
    kc[slot_mapping.long()] = k.to(kc.dtype)
    vc[slot_mapping.long()] = v.to(vc.dtype)


def write_kv_cache(k, v, k_cache, v_cache, slot_mapping, k_scale: float = 1.0, v_scale: float = 1.0):
    """Scatter ``k, v [T, nkv, hd]`` into the paged cache at ``slot_mapping``
    (an fp8 cache stores ``k / k_scale`` and ``v / v_scale``)."""
    if use_native(k):
        ext().write_kv_cache(k, v, k_cache, v_cache, slot_mapping, float(k_scale), float(v_scale))
    else:
        write_kv_cache_ref(k, v, k_cache, v_cache, slot_mapping, k_scale, v_scale)


def paged_decode_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, scale: Optional[float] = None):
    B, nq, hd = q.shape
    nkv = k_cache.shape[2]
    bs = k_cache.shape[1]
    g = nq // nkv
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    out = torch.empty(B, nq, hd, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(seq_lens[b])
        nblk = (L + bs - 1) // bs
        blocks = block_tables[b, :nblk].long()
        kb = k_cache[blocks].reshape(-1, nkv, hd)[:L].float()   # [L, nkv, hd]
        vb = v_cache[blocks].reshape(-1, nkv, hd)[:L].float()
        kb = kb.repeat_interleave(g, dim=1).transpose(0, 1)      # [nq, L, hd]
        vb = vb.repeat_interleave(g, dim=1).transpose(0, 1)
        sc = torch.einsum("hd,hld->hl", q[b].float(), kb) * scale
        out[b] = torch.einsum("hl,hld->hd", torch.softmax(sc, -1), vb)
    return out.to(q.dtype)


def paged_decode_attention(q, k_cache, v_cache, block_tables, seq_lens, scale: Optional[float] = None,
                           max_seq_len: int = 0, k_scale: float = 1.0, v_scale: float = 1.0):
    """One query token per sequence against its paged KV history (``seq_lens``
    includes the token just written).  fp8 caches are dequantised with the
    per-tensor ``k_scale`` / ``v_scale``."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if use_native(q):
        return ext().paged_decode_attn(q, k_cache, v_cache, block_tables, seq_lens, float(scale),
                                       int(max_seq_len), float(k_scale), float(v_scale))
    if k_cache.dtype != q.dtype:
        k_cache = k_cache.to(torch.float32) * k_scale
        v_cache = v_cache.to(torch.float32) * v_scale
    return paged_decode_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, scale)
