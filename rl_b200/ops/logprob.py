"""Fused log-softmax gather / entropy over the vocabulary with an in-place backward.

Replaces the reference's eager vocab-parallel log-softmax path
(``nemo_rl/distributed/model_utils.py``: ``DistributedLogprob`` ``:138``,
``ChunkedDistributedLogprob`` ``:228``, collectives C1-C4; native component N14).

Forward: one pass per row over the (vocab-local) logits computes four
partials with an online softmax - running max ``m``, ``s = sum exp(x/T - m)``,
``u = sum (x/T) exp(x/T - m)`` and the target logit ``x_t/T`` (0 when the
target is not in this shard).  From these, ``logprob = x_t/T - lse`` and
``entropy = lse - u/s`` follow; with tensor parallelism the partials of the
shards are combined with three tiny ``[T]`` all-reduces instead of moving
``[T, V]`` logits.

Backward: ``dlogits = dlogp * (onehot(t) - softmax(x/T)) / T`` written in place
over the bf16 logits buffer, so no fp32 ``[T, V]`` tensor is ever created.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from rl_b200.ops._ext import ext, use_native

__all__ = ["token_logprobs", "token_logprobs_ref", "logits_entropy_ref", "logprob_partials",
           "logprob_partials_ref", "vocab_parallel_logprobs", "token_logprobs_and_entropy"]


def token_logprobs_ref(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    lp = torch.log_softmax(logits.float() / temperature, dim=-1)
    return lp.gather(-1, targets.long().unsqueeze(-1)).squeeze(-1)


def logits_entropy_ref(logits: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    lp = torch.log_softmax(logits.float() / temperature, dim=-1)
    return -(lp.exp() * lp).sum(-1)


def logprob_partials_ref(logits: torch.Tensor, targets_local: torch.Tensor, temperature: float = 1.0):
    x = logits.float() / temperature
    m = x.max(-1).values
    e = torch.exp(x - m.unsqueeze(-1))
    s = e.sum(-1)
    u = (x * e).sum(-1)
    V = x.shape[-1]
    t = targets_local.long()
    inside = (t >= 0) & (t < V)
    xt = torch.where(inside, x.gather(-1, t.clamp(0, V - 1).unsqueeze(-1)).squeeze(-1), torch.zeros_like(m))
    return m, s, u, xt


def logprob_partials(logits: torch.Tensor, targets_local: torch.Tensor, temperature: float = 1.0):
    """Per-row (max, sumexp, sum x*exp, target logit) over this vocab shard, fp32 ``[T]`` each."""
    if use_native(logits):
        return ext().logprob_partials(logits.contiguous(), targets_local.contiguous(), float(temperature))
    return logprob_partials_ref(logits, targets_local, temperature)


def _bwd_inplace(dlp: torch.Tensor, logits: torch.Tensor, targets_local: torch.Tensor, lse: torch.Tensor,
                 temperature: float, out: torch.Tensor) -> torch.Tensor:
    if use_native(logits):
        ext().logprob_bwd(dlp.contiguous().float(), logits, targets_local.contiguous(), lse.contiguous(),
                          float(temperature), out)
        return out
    x = logits.float() / temperature
    p = torch.exp(x - lse.unsqueeze(-1))
    V = x.shape[-1]
    t = targets_local.long()
    inside = (t >= 0) & (t < V)
    g = -p * dlp.unsqueeze(-1)
    rows = torch.arange(x.shape[0], device=x.device)[inside]
    g[rows, t[inside]] += dlp[inside]
    out.copy_((g / temperature).to(out.dtype))
    return out


def _combine(m, s, u, xt, group):
    if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
        gm = m.clone()
        dist.all_reduce(gm, op=dist.ReduceOp.MAX, group=group)
        f = torch.exp(m - gm)
        su = torch.stack([s * f, u * f, xt])
        dist.all_reduce(su, group=group)
        s, u, xt = su[0], su[1], su[2]
        m = gm
    lse = m + torch.log(s)
    return lse, xt - lse, lse - u / s


class _VocabParallelLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, vocab_start, temperature, group, inplace_backward):
        tl = (targets - vocab_start).to(torch.int64)
        m, s, u, xt = logprob_partials(logits, tl, temperature)
        lse, lp, ent = _combine(m, s, u, xt, group)
        ctx.save_for_backward(logits, tl, lse)
        ctx.temperature = temperature
        ctx.inplace = inplace_backward
        ctx.mark_non_differentiable(ent)
        return lp, ent

    @staticmethod
    def backward(ctx, dlp, dent):
        logits, tl, lse = ctx.saved_tensors
        out = logits if ctx.inplace else torch.empty_like(logits)
        _bwd_inplace(dlp, logits, tl, lse, ctx.temperature, out)
        return out, None, None, None, None, None


def vocab_parallel_logprobs(logits: torch.Tensor, targets: torch.Tensor, vocab_start: int = 0,
                            temperature: float = 1.0, group=None, inplace_backward: bool = True):
    """Returns ``(logprobs [T], entropy [T])`` (fp32) of ``targets`` under
    ``softmax(logits/temperature)`` where ``logits`` is this rank's vocab shard
    starting at ``vocab_start``.  Differentiable in ``logprobs``."""
    return _VocabParallelLogprob.apply(logits, targets, vocab_start, float(temperature), group, inplace_backward)


def token_logprobs(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0,
                   inplace_backward: bool = True) -> torch.Tensor:
    return vocab_parallel_logprobs(logits, targets, 0, temperature, None, inplace_backward)[0]


@torch.no_grad()
def token_logprobs_and_entropy(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0,
                               vocab_start: int = 0, group=None):
    tl = (targets - vocab_start).to(torch.int64)
    m, s, u, xt = logprob_partials(logits, tl, temperature)
    lse, lp, ent = _combine(m, s, u, xt, group)
    return lp, ent
