"""Block-scaled fp8 training linear (``megatron_cfg.fp8_cfg: {enabled, fp8: e4m3,
fp8_recipe: blockwise}``).

``y = x @ W^T`` with

* fprop: ``x`` quantised per token and 128-wide K group (1 x 128), ``W`` in
  128 x 128 blocks, block-scaled e4m3 GEMM (``rl_b200.ops.fp8_gemm``);
* dgrad: ``dx = dy @ W`` as the same GEMM on ``dy`` (1 x 128 along the output
  features) and the e4m3 transpose of ``W``, whose 128 x 128 blocks and scales
  are those of ``W`` transposed (no second quantisation);
* wgrad: bf16 product accumulated straight into the fp32 main gradient
  (``dy^T x`` needs 1 x 128 groups along the tokens for both operands, which
  the block-scaled kernels do not take).

Scales are powers of two by default (the tensor cores apply them:
``kind::mxf8f6f4.block_scale``); ``pow2=False`` keeps fp32 scales and the
promoting kernel.  The quantised weight (and its transpose) is cached per
weight and refreshed when the model's ``weight_version`` changes (optimizer
step, reference-policy swap, checkpoint load).

Reference: ``fp8_cfg`` of the reference's Megatron backend
(``examples/configs/grpo_math_1B.yaml:371-375``; recipe notes ``docs/fp8.md``).
"""

from __future__ import annotations

import torch

from rl_b200.ops import gemm as _gemm
from rl_b200.ops.fp8_gemm import gemm_fp8, gemm_mxf8, mx_weight_scales, quant_act_mx
from rl_b200.ops.quant import quant_fp8_block, quant_fp8_group

__all__ = ["Fp8Weight", "fp8_train_linear", "fp8_supported"]


def fp8_supported(w: torch.Tensor) -> bool:
    """Both GEMMs of the layer contract over a multiple of 128 (K for fprop,
    the output features for dgrad)."""
    return w.dim() == 2 and w.shape[0] % 128 == 0 and w.shape[1] % 128 == 0


class Fp8Weight:
    """e4m3 copies of one weight for the forward (``[N, K]``) and the input
    gradient (``[K, N]``), with their block scales."""

    __slots__ = ("version", "pow2", "q", "s", "qt", "st")

    def __init__(self, w: torch.Tensor, version: int, pow2: bool):
        self.version, self.pow2 = version, pow2
        with torch.no_grad():
            q, s = quant_fp8_block(w.detach(), 128, pow2)
            self.q = q
            self.qt = q.view(torch.uint8).t().contiguous().view(torch.float8_e4m3fn)
            s_t = s.t().contiguous()
            if pow2:
                self.s, self.st = mx_weight_scales(s), mx_weight_scales(s_t)
            else:
                self.s, self.st = s, s_t


def _gemm_q(a: torch.Tensor, q: torch.Tensor, s: torch.Tensor, pow2: bool) -> torch.Tensor:
    if pow2:
        aq, as_t = quant_act_mx(a)
        return gemm_mxf8(aq, as_t, q, s)
    aq, as_ = quant_fp8_group(a, 128, False)
    return gemm_fp8(aq, as_, q, s)


class _Fp8LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, fw: Fp8Weight):
        ctx.save_for_backward(x, w)
        ctx.fw = fw
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        y = _gemm_q(x2, fw.q, fw.s, fw.pow2).to(x.dtype)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        fw = ctx.fw
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = _gemm_q(dy2.to(torch.bfloat16) if dy2.is_cuda else dy2, fw.qt, fw.st, fw.pow2)
            dx = dx.to(x.dtype).view(x.shape)
        dw = None
        if ctx.needs_input_grad[1]:
            x2 = x.reshape(-1, x.shape[-1])
            main = getattr(w, "main_grad", None)
            if main is not None:
                _gemm.mm_tn_accumulate(dy2, x2, main)
            else:
                dw = _gemm.mm_tn(dy2, x2).to(w.dtype)
        return dx, dw, None


def fp8_train_linear(x: torch.Tensor, w: torch.Tensor, cache: dict, name: str, version: int,
                     pow2: bool = True) -> torch.Tensor:
    """fp8 linear for weight ``w`` (quantised copies cached in ``cache[name]``
    until ``version`` changes)."""
    fw = cache.get(name)
    if fw is None or fw.version != version or fw.pow2 != pow2:
        fw = cache[name] = Fp8Weight(w, version, pow2)
    return _Fp8LinearFn.apply(x, w, fw)
