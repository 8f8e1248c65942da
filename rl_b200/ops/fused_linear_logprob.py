"""LM-head GEMM fused with the vocab-parallel logprob / entropy, chunked over tokens.

Counterpart of the reference's fused linear cross-entropy
(``ChunkedDistributedHiddenStatesToLogprobs``, ``nemo_rl/distributed/model_utils.py:2572``,
enabled by ``use_fused_linear_logprobs`` / ``fused_linear_logprobs_chunk_size``).

Forward, per chunk of ``chunk`` tokens: ``logits = h_c @ W^T`` (vocab shard), the
fused partials kernel reduces them to (max, sumexp, sum x*exp, target logit),
and the logits chunk is dropped.  Only ``hidden``, the weight and the per-token
log-sum-exp are saved.  Backward, per chunk: recompute the logits, turn them
in place into ``dlogits``, then ``dh_c = dlogits @ W`` and
``W.main_grad += dlogits^T @ h_c``.  Peak extra memory is one ``[chunk, V/tp]``
bf16 tile instead of the full ``[T, V]`` logits (plus their fp32 gradient).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from rl_b200.ops import gemm as _gemm
from rl_b200.ops.logprob import _bwd_inplace, _combine, logprob_partials

__all__ = ["linear_logprobs"]


class _LinearLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, vocab_start, temperature, group, chunk):
        T = hidden.shape[0]
        tl = (targets - vocab_start).to(torch.int64)
        lps, ents, lses = [], [], []
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            logits = _gemm.mm_nt(hidden[s:e], weight)
            m, sm, u, xt = logprob_partials(logits, tl[s:e], temperature)
            del logits
            lse, lp, ent = _combine(m, sm, u, xt, group)
            lps.append(lp)
            ents.append(ent)
            lses.append(lse)
        lp = torch.cat(lps) if lps else hidden.new_zeros(0, dtype=torch.float32)
        ent = torch.cat(ents) if ents else hidden.new_zeros(0, dtype=torch.float32)
        lse = torch.cat(lses) if lses else hidden.new_zeros(0, dtype=torch.float32)
        ctx.save_for_backward(hidden, weight, tl, lse)
        ctx.temperature = temperature
        ctx.chunk = chunk
        ctx.mark_non_differentiable(ent)
        return lp, ent

    @staticmethod
    def backward(ctx, dlp, dent):
        hidden, weight, tl, lse = ctx.saved_tensors
        T = hidden.shape[0]
        chunk = ctx.chunk
        dh = torch.empty_like(hidden)
        main = getattr(weight, "main_grad", None)
        dw = None
        if main is None and ctx.needs_input_grad[1]:
            dw = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
        acc = main if main is not None else dw
        dlp = dlp.float()
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            logits = _gemm.mm_nt(hidden[s:e], weight)
            _bwd_inplace(dlp[s:e], logits, tl[s:e], lse[s:e], ctx.temperature, logits)
            dh[s:e] = _gemm.mm_nn(logits, weight)
            if acc is not None:
                _gemm.mm_tn_accumulate(logits, hidden[s:e], acc)
            del logits
        return dh, (dw.to(weight.dtype) if dw is not None else None), None, None, None, None, None


def linear_logprobs(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, vocab_start: int = 0,
                    temperature: float = 1.0, group=None, chunk: int = 4096):
    """``(logprobs, entropy)`` of ``targets`` under ``softmax(hidden @ weight^T / T)``
    where ``weight`` is this rank's vocab shard; fp32 ``[T]`` each."""
    return _LinearLogprob.apply(hidden, weight, targets, int(vocab_start), float(temperature), group, int(chunk))
