"""Token sampling with temperature / top-k / top-p and the sampled token's logprob
(native component N16; reference: vLLM sampler with
``logprobs_mode: processed_logprobs``, ``examples/configs/grpo_math_1B.yaml:373``,
and train-side ``TrainingSamplingParams`` ``nemo_rl/algorithms/logits_sampling_utils.py:30``).

The CUDA kernel (``csrc/sampling.cu``) samples by the Gumbel-max trick: the
returned token is ``argmax_i(x_i / T + g_i)`` over the kept set, with
``g_i = -log(-log(u_i))`` and ``u_i`` from a counter-based hash of
``(seed, row, i)``; this is an exact draw from ``softmax(x / T)`` restricted to
the kept set and needs one pass over the row (plus a bisection for top-p).
The logprob returned is ``x_tok / T - logsumexp_kept(x / T)``, i.e. the
log-probability under the processed (filtered) distribution.
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.ops._ext import ext, use_native

__all__ = ["sample_tokens", "sample_tokens_ref", "filter_logits_ref"]


def filter_logits_ref(logits: torch.Tensor, temperature: float, top_k: Optional[int], top_p: float) -> torch.Tensor:
    x = logits.float() / max(temperature, 1e-6)
    if top_k is not None and 0 < top_k < x.shape[-1]:
        kth = torch.topk(x, top_k, dim=-1).values[..., -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    if top_p is not None and top_p < 1.0:
        sx, si = torch.sort(x, dim=-1, descending=True)
        p = torch.softmax(sx, -1)
        cum = p.cumsum(-1)
        drop = (cum - p) >= top_p   # keep the smallest prefix whose mass reaches top_p
        sx = sx.masked_fill(drop, float("-inf"))
        x = torch.full_like(x, float("-inf")).scatter(-1, si, sx)
    return x


def sample_tokens_ref(logits: torch.Tensor, temperature: float = 1.0, top_k: Optional[int] = None,
                      top_p: float = 1.0, generator: Optional[torch.Generator] = None):
    x = filter_logits_ref(logits, temperature, top_k, top_p)
    lp = torch.log_softmax(x, -1)
    if temperature <= 0:
        tok = x.argmax(-1)
    else:
        tok = torch.multinomial(lp.exp(), 1, generator=generator).squeeze(-1)
    return tok, lp.gather(-1, tok.unsqueeze(-1)).squeeze(-1)


def sample_tokens(logits: torch.Tensor, temperature: float = 1.0, top_k: Optional[int] = None,
                  top_p: float = 1.0, seed: int = 0, offset: int = 0,
                  out_tokens: Optional[torch.Tensor] = None, out_logprobs: Optional[torch.Tensor] = None,
                  generator: Optional[torch.Generator] = None):
    """Sample one token per row of ``logits [B, V]``; returns ``(tokens int64 [B], logprobs fp32 [B])``.

    ``seed``/``offset`` select the random stream on the native path (``offset``
    is typically the decode step, so a CUDA-graph replay can advance it through
    a device scalar; see ``sample_tokens_graphable``)."""
    if use_native(logits):
        B = logits.shape[0]
        if out_tokens is None:
            out_tokens = torch.empty(B, dtype=torch.int64, device=logits.device)
        if out_logprobs is None:
            out_logprobs = torch.empty(B, dtype=torch.float32, device=logits.device)
        off = torch.tensor([offset], dtype=torch.int64, device=logits.device)
        ext().sample(logits.contiguous(), float(temperature), int(top_k or 0), float(top_p), int(seed), off,
                     out_tokens, out_logprobs)
        return out_tokens, out_logprobs
    return sample_tokens_ref(logits, temperature, top_k, top_p, generator)


def sample_tokens_graphable(logits: torch.Tensor, temperature: float, top_k: Optional[int], top_p: float,
                            seed: int, offset_dev: torch.Tensor, out_tokens: torch.Tensor,
                            out_logprobs: torch.Tensor) -> None:
    """Native sampling whose random offset lives in a device tensor (captured
    into the decode CUDA graph; the kernel advances nothing itself, the caller
    increments ``offset_dev`` between replays)."""
    ext().sample(logits, float(temperature), int(top_k or 0), float(top_p), int(seed), offset_dev,
                 out_tokens, out_logprobs)
