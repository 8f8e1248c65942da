"""Linear layer with gradient-accumulation fusion into fp32 main-grad buffers.

``y = x @ W^T`` with ``W [out, in]``.  In the backward pass the weight gradient
is accumulated straight into ``W.main_grad`` (an fp32 view into the flat
gradient buffer owned by the optimizer) instead of materialising a bf16
``W.grad`` - the equivalent of MCore's ``gradient_accumulation_fusion``
(``examples/configs/grpo_math_1B.yaml``, ``megatron_cfg.gradient_accumulation_fusion``),
so micro-batch accumulation happens in fp32 and the optimizer reads one flat buffer.

GEMMs on CUDA go to ``rl_b200.ops.gemm`` (tcgen05 kernels for the shapes they
cover, the library GEMM otherwise).
"""

from __future__ import annotations

import torch

from rl_b200.ops import gemm as _gemm

__all__ = ["linear", "LinearFn"]


class LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        x2 = x.reshape(-1, x.shape[-1])
        y = _gemm.mm_nt(x2, w)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        x2 = x.reshape(-1, x.shape[-1])
        dx = None
        if ctx.needs_input_grad[0]:
            dx = _gemm.mm_nn(dy2, w).view(x.shape)
        dw = None
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            if main is not None:
                _gemm.mm_tn_accumulate(dy2, x2, main)
            else:
                dw = _gemm.mm_tn(dy2, x2).to(w.dtype)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return LinearFn.apply(x, w)
