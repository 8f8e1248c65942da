"""Block-scaled e4m3 GEMMs (1 x 128 activation scales, 128 x 128 weight scales).

Two kernels in ``csrc/gemm_fp8.cu``:

* ``gemm_fp8(a_q, a_s, b_q, b_s)`` - arbitrary fp32 scales: every 128-wide K
  block is multiplied by tcgen05 ``kind::f8f6f4`` into its own tensor-memory
  accumulator and promoted into fp32 registers with ``a_s[m, kb] * b_s[n/128, kb]``.
* ``gemm_mxf8(a_q, a_s_t, b_q, b_s_t)`` - power-of-two scales, applied by the
  tensor cores (``kind::mxf8f6f4.block_scale`` with UE8M0 scale bytes in tensor
  memory): one accumulator over all of K.  Scales are MN-major
  (``[K/128, rows]``, padded) so the TMA unit fetches each K block's scales with
  its operand tiles; ``quant_act_mx`` and ``mx_weight_scales`` produce them.

On CPU the dequantised fp32 product is the reference for both.

Reference: the 128 x 128 / 1 x 128 block-scaled recipe of the reference's fp8
rollout (``nemo_rl/models/generation/vllm/quantization/fp8.py:756`` weight
blocks, ``:1926`` per-token-group activation quantisation, power-of-two scales
``pow2_weight_scaling_factors`` / ``pow2_activation_scaling_factors`` ``:408-413``)
and its Megatron ``fp8_recipe: blockwise`` training setting
(``examples/configs/grpo_math_1B.yaml:245``).
"""

from __future__ import annotations

import torch

from rl_b200.ops._ext import ext, use_native
from rl_b200.ops.quant import quant_fp8_group, quant_fp8_group_ref

__all__ = ["gemm_fp8", "gemm_fp8_ref", "fp8_linear", "gemm_mxf8", "quant_act_mx", "mx_weight_scales",
           "fp8_linear_mx"]


def gemm_fp8_ref(a_q: torch.Tensor, a_s: torch.Tensor, b_q: torch.Tensor, b_s: torch.Tensor) -> torch.Tensor:
    """fp32 reference of the block-scaled product (same quantised inputs;
    ``a_s [M, K/128]``, ``b_s [ceil(N/128), K/128]``)."""
    M, K = a_q.shape
    N = b_q.shape[0]
    a = a_q.float() * a_s.float().repeat_interleave(128, 1)[:, :K]
    b = b_q.float() * b_s.float().repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)[:, :K]
    return a @ b.t()


def gemm_fp8(a_q: torch.Tensor, a_s: torch.Tensor, b_q: torch.Tensor, b_s: torch.Tensor,
             splits: int = 0) -> torch.Tensor:
    if use_native(a_q):
        return ext().gemm_fp8(a_q.contiguous(), a_s.contiguous(), b_q.contiguous(), b_s.contiguous(), int(splits))
    return gemm_fp8_ref(a_q, a_s, b_q, b_s).to(torch.bfloat16)


def fp8_linear(x: torch.Tensor, w_q: torch.Tensor, w_s: torch.Tensor) -> torch.Tensor:
    """``x [.., K]`` (bf16) times an e4m3 block-scaled weight ``[N, K]`` -> bf16 ``[.., N]``."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    a_q, a_s = quant_fp8_group(x2, 128, False)
    y = gemm_fp8(a_q, a_s, w_q, w_s)
    return y.reshape(*shp[:-1], w_q.shape[0])


# ------------------------------------------------ power-of-two (hardware-scaled)
def quant_act_mx(x: torch.Tensor):
    """1 x 128 e4m3 quantisation with power-of-two scales in the MN-major layout
    ``[K/128, Mp]`` (``Mp`` = rows rounded up to 128; padding scales 1)."""
    if use_native(x):
        return ext().quant_fp8_group_t(x.contiguous(), 128, True)
    q, s = quant_fp8_group_ref(x, 128, True)
    M = x.shape[0]
    Mp = max(128, -(-M // 128) * 128)
    st = torch.ones(s.shape[1], Mp, dtype=torch.float32, device=x.device)
    st[:, :M] = s.t()
    return q, st


def mx_weight_scales(b_s: torch.Tensor) -> torch.Tensor:
    """``[ceil(N/128), K/128]`` power-of-two block scales -> the kernel's MN-major
    padded layout ``[K/128, NBp]`` (done once per weight update)."""
    NB, KB = b_s.shape
    NBp = ((NB + 3) // 4) * 4 + 4
    out = torch.ones(KB, NBp, dtype=torch.float32, device=b_s.device)
    out[:, :NB] = b_s.t()
    return out


def gemm_mxf8(a_q: torch.Tensor, a_s_t: torch.Tensor, b_q: torch.Tensor, b_s_t: torch.Tensor,
              splits: int = 0) -> torch.Tensor:
    if use_native(a_q):
        return ext().gemm_mxf8(a_q.contiguous(), a_s_t, b_q.contiguous(), b_s_t, int(splits))
    M, N = a_q.shape[0], b_q.shape[0]
    NB = -(-N // 128)
    return gemm_fp8_ref(a_q, a_s_t[:, :M].t(), b_q, b_s_t[:, :NB].t()).to(torch.bfloat16)


def fp8_linear_mx(x: torch.Tensor, w_q: torch.Tensor, w_s_t: torch.Tensor) -> torch.Tensor:
    """``x [.., K]`` times a power-of-two block-scaled e4m3 weight (scales from
    ``mx_weight_scales``) -> bf16 ``[.., N]``."""
    shp = x.shape
    a_q, a_s_t = quant_act_mx(x.reshape(-1, shp[-1]))
    y = gemm_mxf8(a_q, a_s_t, w_q, w_s_t)
    return y.reshape(*shp[:-1], w_q.shape[0])
