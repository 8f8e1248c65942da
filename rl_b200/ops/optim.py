"""Fused AdamW over flat fp32 buffers and the gradient-norm reduction.

Replaces the fused Adam of MCore's distributed optimizer (native component N13;
``use_precision_aware_optimizer``, ``examples/configs/grpo_math_1B.yaml:226``).
All master weights, gradients and Adam moments of a model (or of this rank's
shard of it) live in single contiguous fp32 buffers, so one launch updates
everything and also writes the bf16 working copy of the parameters (the
"refit" cast of colocated generation happens in that same pass).
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.ops._ext import ext, use_native

__all__ = ["adamw_step", "adamw_step_ref", "sum_of_squares"]


def adamw_step_ref(master, grad, exp_avg, exp_avg_sq, lr, beta1, beta2, eps, weight_decay, step,
                   grad_scale: float = 1.0, param_out: Optional[torch.Tensor] = None):
    g = grad.float() * grad_scale
    exp_avg.mul_(beta1).add_(g, alpha=1 - beta1)
    exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (exp_avg_sq / bc2).sqrt().add_(eps)
    master.mul_(1 - lr * weight_decay)
    master.addcdiv_(exp_avg, denom, value=-lr / bc1)
    if param_out is not None:
        param_out.copy_(master.to(param_out.dtype))


def adamw_step(master, grad, exp_avg, exp_avg_sq, lr, beta1, beta2, eps, weight_decay, step,
               grad_scale: float = 1.0, param_out: Optional[torch.Tensor] = None):
    """In-place AdamW (decoupled weight decay, bias-corrected) on flat buffers.

    ``grad`` may be fp32 or bf16; ``grad_scale`` folds in gradient clipping and
    loss-scale; ``param_out`` (bf16, same length) receives the cast weights."""
    if use_native(master):
        ext().adamw_step(master, grad, exp_avg, exp_avg_sq, param_out, float(lr), float(beta1), float(beta2),
                         float(eps), float(weight_decay), int(step), float(grad_scale))
    else:
        adamw_step_ref(master, grad, exp_avg, exp_avg_sq, lr, beta1, beta2, eps, weight_decay, step,
                       grad_scale, param_out)


def sum_of_squares(x: torch.Tensor) -> torch.Tensor:
    """fp32 scalar tensor sum(x^2) (device-side, no host sync)."""
    if use_native(x):
        return ext().sum_sq(x)
    return x.float().pow(2).sum()
