"""SwiGLU activation on the fused gate/up projection (native component N9; the
reference enables ``bias_activation_fusion``, ``grpo_math_1B.yaml:183``).

Layout: ``gu = [T, 2F]`` with the gate in columns ``[0, F)`` and the up
projection in ``[F, 2F)`` (the gate and up weight rows are stored concatenated),
``out = silu(gate) * up``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from rl_b200.ops._ext import ext, use_native

__all__ = ["swiglu", "swiglu_ref"]


def swiglu_ref(gu: torch.Tensor) -> torch.Tensor:
    f = gu.shape[-1] // 2
    g = gu[..., :f].float()
    u = gu[..., f:].float()
    return (F.silu(g) * u).to(gu.dtype)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ctx.save_for_backward(gu)
        return ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dout):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(dout.contiguous(), gu)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    if use_native(gu):
        return _SwiGLU.apply(gu)
    return swiglu_ref(gu)
