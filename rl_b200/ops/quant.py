"""Block-scaled FP8 (e4m3) quantisation.

Reference: ``cast_tensor_to_fp8_blockwise`` (``nemo_rl/models/generation/vllm/quantization/fp8.py:756``,
128x128 weight blocks, optional power-of-two scales ``:803-819``) and the Triton
``_per_token_group_quant_fp8`` kernels (``:1926-2047``, 1x128 activation groups;
native components N2-N4 of the survey).

Scale convention: ``x ~= q.float() * scale`` with ``scale = amax / 448`` per
block (``448`` = largest finite e4m3).  With ``pow2_scale`` the scale is rounded
up to a power of two (E8M0-representable), matching the DeepGEMM-style recipe.
"""

from __future__ import annotations

import torch

from rl_b200.ops._ext import ext, use_native

FP8_MAX = 448.0

__all__ = ["quant_fp8_block_ref", "quant_fp8_block", "quant_fp8_group_ref", "quant_fp8_group",
           "dequant_fp8_block", "FP8_MAX"]


def _scale(amax: torch.Tensor, pow2: bool) -> torch.Tensor:
    s = amax.clamp_min(1e-12) / FP8_MAX
    if pow2:
        s = torch.exp2(torch.ceil(torch.log2(s)))
    return s


def quant_fp8_block_ref(w: torch.Tensor, block: int = 128, pow2_scale: bool = False):
    """128x128 block quantisation of a 2-D weight; returns (q e4m3, scales fp32 [ceil(N/b), ceil(K/b)])."""
    N, K = w.shape
    nb, kb = (N + block - 1) // block, (K + block - 1) // block
    pad = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    pad[:N, :K] = w.float()
    blocks = pad.view(nb, block, kb, block)
    amax = blocks.abs().amax(dim=(1, 3))
    s = _scale(amax, pow2_scale)
    q = (blocks / s[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).view(nb * block, kb * block)[:N, :K]
    return q.to(torch.float8_e4m3fn), s


def quant_fp8_group_ref(x: torch.Tensor, group: int = 128, pow2_scale: bool = False):
    """1 x group per-token quantisation; returns (q e4m3 [T, K], scales fp32 [T, K/group])."""
    T, K = x.shape
    assert K % group == 0
    g = x.float().view(T, K // group, group)
    s = _scale(g.abs().amax(-1), pow2_scale)
    q = (g / s[..., None]).clamp(-FP8_MAX, FP8_MAX).view(T, K)
    return q.to(torch.float8_e4m3fn), s


def dequant_fp8_block(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    full = s.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * full


def quant_fp8_block(w: torch.Tensor, block: int = 128, pow2_scale: bool = False, out=None, out_scale=None):
    if use_native(w):
        return ext().quant_fp8_block(w.contiguous(), int(block), bool(pow2_scale), out, out_scale)
    return quant_fp8_block_ref(w, block, pow2_scale)


def quant_fp8_group(x: torch.Tensor, group: int = 128, pow2_scale: bool = False):
    if use_native(x):
        return ext().quant_fp8_group(x.contiguous(), int(group), bool(pow2_scale))
    return quant_fp8_group_ref(x, group, pow2_scale)
