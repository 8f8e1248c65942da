"""LM-head GEMM fused with the vocab-parallel logprob / entropy, chunked over tokens.

Counterpart of the reference's fused linear cross-entropy
(``ChunkedDistributedHiddenStatesToLogprobs``, ``nemo_rl/distributed/model_utils.py:2572``,
enabled by ``use_fused_linear_logprobs`` / ``fused_linear_logprobs_chunk_size``).

On CUDA both passes are one tcgen05 GEMM each (``csrc/gemm_sm100.cu``):

* forward: the LM-head product's epilogue reduces every 256-column logits tile
  in tensor memory to per-row online-softmax partials (max, sum exp, sum x exp)
  and the target's logit; a small kernel merges the tiles.  No logits reach
  HBM: the traffic is the weight, the hidden states and 12 bytes per row per
  256 vocabulary columns of partials.
* backward: the same product recomputes each tile and its epilogue writes
  ``dlogits = dlogp / T * (onehot - softmax)`` as bf16, which feeds the dgrad
  (``dh_c = dlogits @ W``) and wgrad (``W.main_grad += dlogits^T @ h_c``)
  products directly.

Elsewhere (CPU) the chunked reference path materialises one ``[chunk, V/tp]``
logits tile at a time.  Only ``hidden``, the weight and the per-token
log-sum-exp are saved for the backward.  Under tensor parallelism the per-row
partials of the shards are combined (max, then rescaled sums) over the group.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from rl_b200.ops import gemm as _gemm
from rl_b200.ops._ext import ext, use_native
from rl_b200.ops.logprob import _bwd_inplace, _combine, logprob_partials

__all__ = ["linear_logprobs"]

# Tokens per fused forward launch: no logits tile is kept, only 12 bytes of
# partials per row per 256 vocabulary columns (~6 KB per token at V = 128K).
FUSED_FWD_CHUNK = 16384


def _fused_ok(hidden: torch.Tensor, weight: torch.Tensor) -> bool:
    """The tcgen05 LM-head kernels take bf16 [T, H] x [V, H] with H % 8 == 0."""
    return (use_native(hidden) and hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and hidden.dim() == 2 and hidden.shape[1] % 8 == 0 and weight.is_contiguous()
            and hidden.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0)


class _LinearLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, targets, vocab_start, temperature, group, chunk):
        T = hidden.shape[0]
        tl = (targets - vocab_start).to(torch.int64).contiguous()
        fused = _fused_ok(hidden, weight)
        if fused:
            hidden = hidden.contiguous()
        step = max(chunk, FUSED_FWD_CHUNK) if fused else chunk
        lps, ents, lses = [], [], []
        for s in range(0, T, step):
            e = min(T, s + step)
            if fused:
                m, sm, u, xt = ext().gemm_logprob_partials(hidden[s:e], weight, tl[s:e], float(temperature))
            else:
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
        dlp = dlp.float().contiguous()
        fused = _fused_ok(hidden, weight)
        for s in range(0, T, chunk):
            e = min(T, s + chunk)
            if fused:
                logits = ext().gemm_dlogits(hidden[s:e], weight, tl[s:e], lse[s:e].contiguous(), dlp[s:e],
                                            float(ctx.temperature))
            else:
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


def filter_logits_top_k_top_p(logits: torch.Tensor, top_k: Optional[int], top_p: float) -> torch.Tensor:
    """Mask (to -inf) everything outside the top-k / nucleus-p set of each row,
    the same filter the rollout sampler applies (ties at the k-th value kept)."""
    if top_k:
        kth = torch.topk(logits, min(int(top_k), logits.shape[-1]), dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    if top_p is not None and top_p < 1.0:
        srt, idx = torch.sort(logits, dim=-1, descending=True)
        cum = torch.softmax(srt, -1).cumsum(-1)
        drop = (cum - torch.softmax(srt, -1)) >= top_p  # keep the smallest prefix reaching top_p
        mask = torch.zeros_like(drop).scatter(-1, idx, drop)
        logits = logits.masked_fill(mask, float("-inf"))
    return logits


def filtered_linear_logprobs(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, vocab_start: int,
                             temperature: float, top_k: Optional[int], top_p: float, group=None,
                             chunk: int = 1024):
    """Training-time log-probabilities under the rollout's top-k / top-p filter
    (renormalised over the kept tokens), so the ratio in the policy loss compares
    like with like.  Reference: ``TrainingSamplingParams`` / ``apply_top_k_top_p``
    (``nemo_rl/algorithms/logits_sampling_utils.py:30,256``).  The vocab shards are
    all-gathered per chunk of tokens (the filter needs whole rows); returns
    (logprob [T], entropy [T]) of the filtered distribution."""
    from rl_b200.parallel.comm import gather_from_sp

    lps, ents = [], []
    for s in range(0, hidden.shape[0], chunk):
        e = min(hidden.shape[0], s + chunk)
        logits = torch.matmul(hidden[s:e], weight.t()).float()
        if group is not None and dist.get_world_size(group) > 1:
            logits = gather_from_sp(logits.t().contiguous(), group).t()
        logits = filter_logits_top_k_top_p(logits / temperature, top_k, top_p)
        logp = torch.log_softmax(logits, -1)
        lps.append(logp.gather(1, targets[s:e].long().unsqueeze(1)).squeeze(1))
        p = logp.exp()
        ents.append(-(p * torch.where(p > 0, logp, torch.zeros_like(logp))).sum(-1))
    return torch.cat(lps), torch.cat(ents)
