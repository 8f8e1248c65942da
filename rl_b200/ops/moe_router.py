"""MoE router: softmax over the experts, top-k and the expert-grouped permutation.

Replaces the router top-k and token permutation of Transformer Engine's MoE path
(the reference patches TE's permutation kernel, ``nemo_rl/models/policy/workers/patches.py:56``).
On CUDA the three kernels of ``csrc/moe_router.cu`` produce, from fp32 logits,
the probabilities, the top-k expert ids (ties go to the lower id), the tokens
per expert and the stable expert-grouped order of the ``T * k`` assignments
(the order ``torch.argsort(ids.flatten(), stable=True)`` gives), so the MoE
block needs no sort, histogram or top-k of its own.  The gradient reaches the
logits through the softmax (the selection is piecewise constant).
"""

from __future__ import annotations

import torch

from rl_b200.ops._ext import ext

__all__ = ["router_topk", "router_topk_ref"]


def router_topk_ref(logits: torch.Tensor, k: int):
    """fp32 PyTorch path: (probs [T, E], ids [T, k] int64, counts [E] int32,
    order [T*k] int64)."""
    probs = torch.softmax(logits.float(), -1)
    ids = torch.topk(probs, k, dim=-1)[1]
    flat = ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=logits.shape[-1]).to(torch.int32)
    return probs, ids, counts, order


class _RouterTopK(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, k):
        probs, ids, counts, order, _pos = ext().moe_router_topk(logits.contiguous(), int(k))
        ctx.save_for_backward(probs)
        ctx.mark_non_differentiable(ids, counts, order)
        return probs, ids, counts, order

    @staticmethod
    def backward(ctx, dprobs, _ids, _counts, _order):
        (p,) = ctx.saved_tensors
        if dprobs is None:
            return None, None
        dprobs = dprobs.float()
        return p * (dprobs - (dprobs * p).sum(-1, keepdim=True)), None


# tests switch this off to compare the native router with the PyTorch one on the same GPU
NATIVE = True


def router_topk(logits: torch.Tensor, k: int):
    """``logits [T, E]`` fp32 -> (probs, ids, counts, order); see the module doc."""
    if NATIVE and logits.is_cuda and logits.dtype == torch.float32 and logits.shape[-1] <= 1024 and k <= 64:
        return _RouterTopK.apply(logits, k)
    return router_topk_ref(logits, k)
