"""Rotary position embedding (native component N8; reference enables TE's fused RoPE
with ``apply_rope_fusion: True``, ``examples/configs/grpo_math_1B.yaml:181``).

``apply_rope_qkv`` takes the packed QKV projection ``[T, (nq + 2*nkv) * hd]`` and
returns a tensor of the same shape with the q and k heads rotated (half-split
"rotate_half" convention used by Llama / Qwen HF checkpoints) and v copied, so
the attention kernels read q, k and v from one buffer with strides.

The cos/sin table is built once per model in fp32 from ``inv_freq`` (with the
Llama-3.1 frequency scaling or YaRN when requested) and indexed by position on
device.

YaRN (Peng et al., "YaRN: Efficient Context Window Extension of Large
Language Models", arXiv:2309.00071): with scale ``s = factor`` and original
context ``L``, a frequency that turns more than ``beta_fast`` times over ``L``
keeps its value, one that turns fewer than ``beta_slow`` times is divided by
``s`` (interpolation), and the band in between blends linearly over the
rotary dimension index (the dimension at which a frequency makes ``n`` turns
over ``L`` is ``d ln(L / (2 pi n)) / (2 ln theta)``; ``truncate`` rounds the
band's ends outwards to whole dimensions).  Attention logits are sharpened
by ``t^-1 = (0.1 ln s + 1)^2``, applied as a factor ``0.1 m ln s + 1`` on
cos / sin (so on q and k), divided by the same expression with
``mscale_all_dim`` when that is non-zero.  Reference: YaRN through
``policy.hf_config_overrides.rope_scaling`` (``docs/guides/yarn-long-context.md``;
required fields validated in ``nemo_rl/models/megatron/setup.py``).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from rl_b200.ops._ext import ext, use_native

__all__ = ["rope_inv_freq", "rope_attention_factor", "YARN_FIELDS", "build_rope_cache", "apply_rope_qkv", "apply_rope_qkv_ref", "rotate_half"]


def rope_inv_freq(head_dim: int, theta: float, scaling: Optional[dict] = None) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling and scaling.get("rope_type", scaling.get("type")) == "llama3":
        factor = float(scaling["factor"])
        lo = float(scaling.get("low_freq_factor", 1.0))
        hi = float(scaling.get("high_freq_factor", 4.0))
        old_ctx = float(scaling.get("original_max_position_embeddings", 8192))
        lo_wl, hi_wl = old_ctx / lo, old_ctx / hi
        wl = 2 * math.pi / inv
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        smooth = (old_ctx / wl - lo) / (hi - lo)
        mid = (1 - smooth) * scaled / factor + smooth * scaled
        is_mid = (wl <= lo_wl) & (wl >= hi_wl)
        inv = torch.where(is_mid, mid, scaled)
    elif scaling and scaling.get("rope_type", scaling.get("type")) == "yarn":
        inv = _yarn_inv_freq(inv, head_dim, float(scaling.get("rope_theta", theta)), scaling)
    return inv.to(torch.float32)


YARN_FIELDS = ("rope_type", "rope_theta", "factor", "original_max_position_embeddings", "truncate",
               "beta_fast", "beta_slow", "mscale", "mscale_all_dim")


def _yarn_inv_freq(inv: torch.Tensor, head_dim: int, theta: float, sc: dict) -> torch.Tensor:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    s = float(sc["factor"])
    L = float(sc["original_max_position_embeddings"])

    def dim_at(turns: float) -> float:  # rotary dimension that makes `turns` turns over L
        return head_dim * math.log(L / (turns * 2 * math.pi)) / (2 * math.log(theta))

    lo, hi = dim_at(float(sc.get("beta_fast", 32))), dim_at(float(sc.get("beta_slow", 1)))
    if sc.get("truncate", True):
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, head_dim - 1)
    if hi == lo:
        hi += 0.001
    ramp = ((torch.arange(head_dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
    keep = 1.0 - ramp  # 1: original frequency, 0: interpolated by s
    return inv / s * (1.0 - keep) + inv * keep


def _mscale(s: float, m: float) -> float:
    return 1.0 if s <= 1 else 0.1 * m * math.log(s) + 1.0


def rope_attention_factor(scaling: Optional[dict]) -> float:
    """Factor on cos / sin (1 except for YaRN)."""
    if not scaling or scaling.get("rope_type", scaling.get("type")) != "yarn":
        return 1.0
    if scaling.get("attention_factor") is not None:
        return float(scaling["attention_factor"])
    s = float(scaling["factor"])
    m, m_all = float(scaling.get("mscale") or 1.0), float(scaling.get("mscale_all_dim") or 0.0)
    if m and m_all:
        return _mscale(s, m) / _mscale(s, m_all)
    return _mscale(s, m)


def build_rope_cache(max_pos: int, head_dim: int, theta: float, scaling: Optional[dict] = None,
                     device=None) -> torch.Tensor:
    """``[max_pos, head_dim]`` fp32 table: first half cos, second half sin."""
    inv = rope_inv_freq(head_dim, theta, scaling)
    t = torch.arange(max_pos, dtype=torch.float32)
    ang = torch.outer(t, inv)
    a = rope_attention_factor(scaling)
    return (torch.cat([ang.cos(), ang.sin()], dim=-1) * a).to(device)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope_qkv_ref(qkv: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor, nq: int, nkv: int,
                       hd: int, inverse: bool = False) -> torch.Tensor:
    T = qkv.shape[0]
    x = qkv.float().view(T, nq + 2 * nkv, hd)
    cs = cache[positions.long()]
    cos = torch.cat([cs[:, : hd // 2]] * 2, -1).unsqueeze(1)
    sin = torch.cat([cs[:, hd // 2:]] * 2, -1).unsqueeze(1)
    if inverse:
        sin = -sin
    qk = x[:, : nq + nkv]
    qk = qk * cos + rotate_half(qk) * sin
    out = torch.cat([qk, x[:, nq + nkv:]], dim=1)
    return out.reshape(qkv.shape).to(qkv.dtype)


class _RopeQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, positions, cache, nq, nkv, hd):
        out = ext().rope_qkv(qkv.contiguous(), positions, cache, nq, nkv, hd, False)
        ctx.save_for_backward(positions, cache)
        ctx.dims = (nq, nkv, hd)
        return out

    @staticmethod
    def backward(ctx, dout):
        positions, cache = ctx.saved_tensors
        nq, nkv, hd = ctx.dims
        dqkv = ext().rope_qkv(dout.contiguous(), positions, cache, nq, nkv, hd, True)
        return dqkv, None, None, None, None, None


def apply_rope_qkv(qkv: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor, nq: int, nkv: int,
                   hd: int) -> torch.Tensor:
    if use_native(qkv):
        return _RopeQKV.apply(qkv, positions, cache, nq, nkv, hd)
    return apply_rope_qkv_ref(qkv, positions, cache, nq, nkv, hd)
