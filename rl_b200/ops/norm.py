"""RMSNorm and fused residual-add + RMSNorm with autograd.

Replaces the Transformer-Engine norm kernels the reference trains with (native
component N7 of the survey; called through MCore layers built in
``nemo_rl/models/megatron/setup.py:2520``).  On CUDA tensors the forward and
backward run in ``csrc/norm.cu``; the backward produces ``dx`` and a per-block
fp32 partial of ``dw`` that is reduced in the same launch sequence.
"""

from __future__ import annotations

import torch

from rl_b200.ops._ext import ext, use_native

__all__ = ["rms_norm", "add_rms_norm", "rms_norm_ref", "add_rms_norm_ref"]


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype)


def add_rms_norm_ref(x: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float):
    s = (x.float() + delta.float()).to(x.dtype)
    return rms_norm_ref(s, w, eps), s


def _weight_grad(w: torch.Tensor, dw_fp32: torch.Tensor):
    """Accumulate the fp32 weight gradient straight into ``w.main_grad`` when the
    optimizer attached one (no bf16 ``.grad`` round trip); else return it."""
    main = getattr(w, "main_grad", None)
    if main is not None:
        main.add_(dw_fp32.view_as(main))
        return None
    return dw_fp32.to(w.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y, rstd = ext().rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dx, dw = ext().rmsnorm_bwd(dy.reshape(x2.shape).contiguous(), x2, w, rstd)
        return dx.view(ctx.shape), _weight_grad(w, dw), None


class _AddRMSNorm(torch.autograd.Function):
    """(y, s) = (rmsnorm(x + delta), x + delta): the residual add of one sub-layer
    fused with the normalisation that opens the next."""

    @staticmethod
    def forward(ctx, x, delta, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        d2 = delta.reshape(-1, shape[-1]).contiguous()
        y, s, rstd = ext().add_rmsnorm_fwd(x2, d2, w, eps)
        ctx.save_for_backward(s, w, rstd)
        ctx.shape = shape
        return y.view(shape), s.view(shape)

    @staticmethod
    def backward(ctx, dy, ds):
        s, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(s.shape).contiguous()
        ds2 = None if ds is None else ds.reshape(s.shape).contiguous()
        dx, dw = ext().rmsnorm_bwd_add(dy2, s, w, rstd, ds2)
        dx = dx.view(ctx.shape)
        return dx, dx, _weight_grad(w, dw), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    if use_native(x):
        return _RMSNorm.apply(x, w, eps)
    return rms_norm_ref(x, w, eps)


def add_rms_norm(x: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float = 1e-5):
    """Return ``(rmsnorm(x + delta) * w, x + delta)``."""
    if use_native(x):
        return _AddRMSNorm.apply(x, delta, w, eps)
    return add_rms_norm_ref(x, delta, w, eps)
