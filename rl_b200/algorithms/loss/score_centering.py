"""Score centering for policy-gradient losses (top-k estimator).

The REINFORCE gradient ``A * grad log p(y)`` has the sampler-expected score
``E_{v ~ sampler}[grad log p_v]`` as its drift; subtracting ``A`` times an
estimate of it centres the estimator.  With the sampler's top-k head known
exactly (ids and log-probs ``q`` recorded at rollout time) and the tail modelled
as the trainer's own tail scaled by ``rho = (1 - sum q) / (1 - sum p)``, the
expected score is ``sum_v m_v grad log p_v`` over the head with
``m_v = mass_v - alpha * p_v`` (``sum_v p_v grad log p_v = 0`` turns the tail
term into ``-alpha * p_v`` on the head ids).  Per importance-sampling mode:

* off:   mass = q,                          alpha = rho
* is:    mass = p,                          alpha = 1     (coefficient 0)
* tis:   mass = clamp(p, lo q, hi q),       alpha = clamp(1, lo rho, hi rho)
* icepop: mass = p where lo <= p/q <= hi,   alpha = [lo <= 1/rho <= hi]

The returned per-token term is ``sum_v sg(m_v) log p_v``; the loss adds
``A * term`` (token- or sequence-normalised like the actor loss).

Reference: ``compute_score_centering_term``
(``nemo_rl/algorithms/loss/score_centering.py``) and its use in
``ClippedPGLossFn`` (``nemo_rl/algorithms/loss/loss_functions.py:1071``).
"""

from __future__ import annotations

from typing import Optional

import torch

__all__ = ["score_centering_term"]


def score_centering_term(policy_lp_topk: torch.Tensor, sampler_lp_topk: torch.Tensor, mode: str,
                         bounds: Optional[tuple], mask: torch.Tensor):
    """``policy_lp_topk`` (with grad) and ``sampler_lp_topk`` are ``[B, S, k]``
    log-probs at the sampler's top-k ids; ``mask [B, S]``.  Returns the term
    ``[B, S]`` and the sampler head mass ``[B, S]`` (zero where masked)."""
    act = mask.bool()
    zero = torch.zeros((), dtype=policy_lp_topk.dtype, device=policy_lp_topk.device)
    lp = torch.where(act.unsqueeze(-1), policy_lp_topk, zero)
    lq = torch.where(act.unsqueeze(-1), sampler_lp_topk.detach().to(lp.dtype), zero)
    p, q = lp.detach().exp(), lq.exp()
    head = q.sum(-1)
    rho = (1.0 - head).clamp_min(0.0) / (1.0 - p.sum(-1)).clamp_min(1e-6)
    if mode == "off":
        mass, alpha = q, rho
    elif mode == "is":
        mass, alpha = p, torch.ones_like(rho)
    elif mode == "tis":
        lo, hi = bounds
        mass = torch.minimum(torch.maximum(p, lo * q), hi * q)
        alpha = torch.minimum(torch.maximum(torch.ones_like(rho), lo * rho), hi * rho)
    elif mode == "icepop":
        lo, hi = bounds
        r = (lp.detach() - lq).exp()
        mass = torch.where((r >= lo) & (r <= hi), p, torch.zeros_like(p))
        inv = rho.reciprocal()
        alpha = ((inv >= lo) & (inv <= hi)).to(p.dtype)
    else:
        raise ValueError(f"score centering does not support importance-sampling mode {mode!r}")
    coef = (mass - alpha.unsqueeze(-1) * p).detach()
    term = (coef * lp).sum(-1)
    return torch.where(act, term, zero), torch.where(act, head, zero)
