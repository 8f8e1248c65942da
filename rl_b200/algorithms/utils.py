"""Shared RL math: masked reductions, KL estimators, per-prompt baselines, metrics.

Semantics follow the reference (``nemo_rl/algorithms/utils.py``): ``calculate_kl``
``:56`` (Schulman's k1/k2/k3 estimators with input/output clamps and optional
importance weights), ``calculate_baseline_and_std_per_prompt`` ``:118``
(leave-one-out baseline, unbiased std, trivial-group detection), ``masked_mean``
``:294`` and ``print_performance_metrics`` ``:605``.

The per-prompt statistics here are computed with scatter/segment reductions over
group ids (one pass, no Python loop over prompts), which keeps the driver step
O(batch) on large rollouts.
"""

from __future__ import annotations

import math
from typing import Optional, Union

import torch

__all__ = [
    "masked_mean",
    "calculate_kl",
    "calculate_baseline_and_std_per_prompt",
    "compute_seq_logprob_errors",
    "set_seed",
    "group_ids_from_prompts",
]


def masked_mean(
    values: torch.Tensor,
    mask: torch.Tensor,
    dim: Optional[int] = None,
    global_normalization_factor: Optional[Union[torch.Tensor, float]] = None,
) -> torch.Tensor:
    """``sum(values*mask) / (norm + 1e-8)`` where ``norm`` is ``sum(mask)`` unless a
    global (all-rank) count is supplied, so micro-batch losses add up to the global mean."""
    norm = mask.sum(dim=dim) if global_normalization_factor is None else global_normalization_factor
    return (values * mask).sum(dim=dim) / (norm + 1e-8)


def calculate_kl(
    logprobs: torch.Tensor,
    logprobs_reference: torch.Tensor,
    kl_type: str = "k3",
    input_clamp_value: Optional[float] = 20.0,
    output_clamp_value: Optional[float] = 10.0,
    importance_sampling_weights: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Per-token KL(pi || pi_ref) estimate from sampled-token log-probabilities.

    With ``log_r = logp_ref - logp``: k1 = -log_r, k2 = log_r^2 / 2,
    k3 = exp(log_r) - 1 - log_r (http://joschu.net/blog/kl-approx.html).
    Where the input clamp is active, the importance weight is detached so the
    clamp removes its gradient too.
    """
    log_r = logprobs_reference - logprobs
    w = importance_sampling_weights
    if input_clamp_value is not None:
        clamped = log_r.clamp(-input_clamp_value, input_clamp_value)
        if w is not None:
            w = torch.where(clamped == log_r, w, w.detach())
        log_r = clamped
    if kl_type == "k1":
        kl = -log_r
    elif kl_type == "k2":
        kl = 0.5 * log_r * log_r
    elif kl_type == "k3":
        kl = torch.expm1(log_r) - log_r
    else:
        raise ValueError(f"unknown kl_type {kl_type!r} (expected k1, k2 or k3)")
    if w is not None:
        kl = w * kl
    if output_clamp_value is not None:
        kl = kl.clamp(-output_clamp_value, output_clamp_value)
    return kl


def group_ids_from_prompts(prompts: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Map rows of a ``[B]`` or ``[B, k]`` key tensor to dense group ids."""
    if prompts.dim() == 1:
        prompts = prompts.unsqueeze(-1)
    _, inverse = torch.unique(prompts, dim=0, return_inverse=True)
    return inverse, int(inverse.max().item()) + 1 if inverse.numel() else 0


def calculate_baseline_and_std_per_prompt(
    prompts: torch.Tensor,
    rewards: torch.Tensor,
    valid_mask: torch.Tensor,
    leave_one_out_baseline: bool = True,
    std_rewards: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Baseline, std and "trivial group" flag for each row of a GRPO batch.

    Rows are grouped by equal ``prompts`` keys.  For a row i in a group G with
    valid rows V (``valid_mask``):

    * baseline_i = mean of rewards over V (excluding i itself when
      ``leave_one_out_baseline``), std_i is the unbiased std built from the same
      (leave-one-out) first and second moments;
    * groups with <= 1 valid row get baseline = reward (zero advantage) and std 0;
    * trivial_i is True when every compared reward in the group is equal, so
      normalisation never amplifies float32 rounding noise.
    """
    if std_rewards is None:
        std_rewards = rewards
    device = rewards.device
    gid, G = group_ids_from_prompts(prompts.to(device))
    v = valid_mask.to(device=device, dtype=rewards.dtype)
    loo = 1.0 if leave_one_out_baseline else 0.0

    def seg_sum(x: torch.Tensor) -> torch.Tensor:
        return torch.zeros(G, dtype=x.dtype, device=device).index_add_(0, gid, x)

    n_valid = seg_sum(v)[gid]                      # valid rows in my group
    s1 = seg_sum(rewards * v)[gid]
    s1_std = seg_sum(std_rewards * v)[gid]
    s2 = seg_sum(std_rewards * std_rewards * v)[gid]
    # Remove my own contribution for the leave-one-out estimate (only if I am valid;
    # the reference's (1 - I) mask also removes invalid self rows, whose reward*valid is 0).
    self_r = rewards * v
    self_rs = std_rewards * v
    denom = n_valid - loo
    base = (s1 - loo * self_r) / denom
    base_std = (s1_std - loo * self_rs) / denom
    sq = (s2 - loo * self_rs * std_rewards) / denom
    var = (sq - base_std * base_std) * (denom / (denom - 1))
    std = var.clamp_min(0).sqrt().nan_to_num(0.0)
    # Guard: where var is negative only by rounding, sqrt(clamp) is 0 already.

    degenerate = n_valid <= 1
    baseline = torch.where(degenerate, rewards, base)
    std = torch.where(degenerate, torch.zeros_like(std), std)

    # Trivial distribution: min == max over the compared set (valid rows, minus self
    # under leave-one-out).  Compute group min/max of valid rewards, and the second
    # extreme to handle leave-one-out exclusion of the row itself.
    big = torch.finfo(std_rewards.dtype).max
    vb = v.bool()
    r_for_min = torch.where(vb, std_rewards, torch.full_like(std_rewards, big))
    r_for_max = torch.where(vb, std_rewards, torch.full_like(std_rewards, -big))
    gmin = torch.full((G,), big, dtype=std_rewards.dtype, device=device).scatter_reduce(0, gid, r_for_min, "amin")
    gmax = torch.full((G,), -big, dtype=std_rewards.dtype, device=device).scatter_reduce(0, gid, r_for_max, "amax")
    if leave_one_out_baseline:
        # With self excluded, the group is trivial iff all OTHER valid rewards are equal.
        # Count how many valid rows attain min / max.
        at_min = seg_sum((vb & (std_rewards == gmin[gid])).to(rewards.dtype))[gid]
        at_max = seg_sum((vb & (std_rewards == gmax[gid])).to(rewards.dtype))[gid]
        others = n_valid - v
        # others' min equals others' max iff all others share one value: either
        # the whole group is constant, or I am the unique outlier at min or max.
        whole_const = gmin[gid] == gmax[gid]
        i_unique_min = vb & (std_rewards == gmin[gid]) & (at_min == 1) & (at_max == others)
        i_unique_max = vb & (std_rewards == gmax[gid]) & (at_max == 1) & (at_min == others)
        trivial = whole_const | i_unique_min | i_unique_max
    else:
        trivial = gmin[gid] == gmax[gid]
    trivial = torch.where(degenerate, torch.ones_like(trivial), trivial)
    return baseline, std, trivial


def compute_seq_logprob_errors(
    policy_logprobs: torch.Tensor,
    generation_logprobs: torch.Tensor,
    token_mask: torch.Tensor,
    sample_mask: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-sequence mean of exp(|logp_gen - logp_policy|) over valid tokens (the
    multiplicative probability error that ``seq_logprob_error_threshold`` filters on)."""
    mask = token_mask * sample_mask.unsqueeze(-1)
    counts = mask.sum(-1)
    err = torch.where(mask.bool(), (generation_logprobs - policy_logprobs).abs(), torch.zeros_like(policy_logprobs))
    errors = (torch.exp(err) * mask).sum(-1) / counts.clamp_min(1)
    return errors, counts > 0


def set_seed(seed: int) -> None:
    import random

    import numpy as np

    random.seed(seed)
    np.random.seed(seed % (2**32))
    torch.manual_seed(seed)


def nan_safe(x: float) -> float:
    return 0.0 if (x is None or (isinstance(x, float) and math.isnan(x))) else x
