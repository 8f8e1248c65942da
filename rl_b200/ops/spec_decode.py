"""Speculative decoding: verification of draft tokens against the target model.

``spec_verify(target_logits [B, k+1, V], draft_logits [B, k, V], draft_tokens [B, k])``
returns ``(tokens [B, k+1], n_emit [B], logprobs [B, k+1])``: the accepted draft
prefix followed by one correction (on the first rejection) or bonus token, so
``n_emit`` is between 1 and k+1; slots past the end hold -1.  Sampling is the
standard rejection scheme (accept x with probability min(1, p(x)/q(x)); on
rejection draw from norm(max(0, p - q)); all accepted: draw from p_k), which
leaves the output distributed exactly as plain sampling from the target;
temperature 0 is greedy verification.  ``logprobs`` are the target's
log-probabilities of the emitted tokens (what the trainer compares against).

Reference: vLLM's rejection sampler behind ``speculative_config`` (Eagle3 / MTP
drafts, ``docs/guides/eagle3-speculative-decoding.md``).  Native kernel:
``csrc/spec_decode.cu``; ``spec_verify_ref`` is the torch path (CPU) and test oracle.
"""

from __future__ import annotations

import torch

from rl_b200.ops._ext import ext, use_native

__all__ = ["spec_verify", "spec_verify_ref"]


def spec_verify_ref(target_logits, draft_logits, draft_tokens, temperature: float = 1.0,
                    generator: torch.Generator | None = None):
    B, k1, V = target_logits.shape
    k = k1 - 1
    tok = torch.full((B, k1), -1, dtype=torch.long)
    lp = torch.zeros(B, k1)
    n = torch.zeros(B, dtype=torch.int32)
    greedy = temperature <= 0
    t = target_logits.float().cpu() / (1.0 if greedy else temperature)
    d = draft_logits.float().cpu() / (1.0 if greedy else temperature)
    logp = torch.log_softmax(t, -1)
    for b in range(B):
        for i in range(k1):
            if i == k:
                x = int(t[b, i].argmax()) if greedy else int(torch.multinomial(logp[b, i].exp(), 1, generator=generator))
                tok[b, i], lp[b, i] = x, logp[b, i, x]
                n[b] = i + 1
                break
            x = int(draft_tokens[b, i])
            if greedy:
                y = int(t[b, i].argmax())
                tok[b, i], lp[b, i] = y, logp[b, i, y]
                if y != x:
                    n[b] = i + 1
                    break
                continue
            p = logp[b, i].exp()
            q = torch.softmax(d[b, i], -1)
            u = float(torch.rand(1, generator=generator))
            if u < float(p[x] / q[x]):
                tok[b, i], lp[b, i] = x, logp[b, i, x]
                continue
            r = (p - q).clamp_min(0)
            y = int(torch.multinomial(r / r.sum(), 1, generator=generator)) if r.sum() > 0 else x
            tok[b, i], lp[b, i] = y, logp[b, i, y]
            n[b] = i + 1
            break
    return tok, n, lp


def spec_verify(target_logits, draft_logits, draft_tokens, temperature: float = 1.0, seed: int = 0,
                offset: int = 0):
    if use_native(target_logits):
        return ext().spec_verify(target_logits.contiguous(), draft_logits.contiguous(),
                                 draft_tokens.to(torch.long).contiguous(), float(temperature), int(seed), int(offset))
    g = torch.Generator().manual_seed(int(seed) * 1000003 + int(offset))
    return spec_verify_ref(target_logits, draft_logits, draft_tokens, temperature, g)
