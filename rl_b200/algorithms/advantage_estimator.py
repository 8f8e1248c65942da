"""Advantage estimators (reference: ``nemo_rl/algorithms/advantage_estimator.py``).

* ``GRPOAdvantageEstimator`` (``:106``): reward minus (leave-one-out) group mean,
  divided by the group std where the group is non-trivial.
* ``GDPOAdvantageEstimator`` (``:148``): GRPO per named reward component
  (``reward/<name>`` keys), weighted sum, then batch whitening.
* ``ReinforcePlusPlusAdvantageEstimator`` (``:253``): optional group-mean
  baseline, optional KL-in-reward, global token whitening.
* ``RawRewardAdvantageEstimator``: reward as advantage, optional whitening.
* ``GeneralizedAdvantageEstimator`` (``:381``): GAE(gamma, lambda) over a value
  model's per-token values with carry-forward masking (masked positions keep the
  running accumulators so prompt / padding tokens add no phantom TD error).
* ``OPDAdvantageEstimator``: on-policy distillation, per-token advantage =
  log of the (proximal) teacher mixture minus the student log-probability.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from rl_b200.algorithms.utils import calculate_baseline_and_std_per_prompt, calculate_kl, masked_mean

__all__ = [
    "GRPOAdvantageEstimator",
    "GDPOAdvantageEstimator",
    "ReinforcePlusPlusAdvantageEstimator",
    "RawRewardAdvantageEstimator",
    "GeneralizedAdvantageEstimator",
    "OPDAdvantageEstimator",
    "make_advantage_estimator",
]


def _masked_var(x: torch.Tensor, mask: torch.Tensor, mean: torch.Tensor) -> torch.Tensor:
    n = mask.sum()
    return ((x - mean) ** 2 * mask).sum() / (n - 1).clamp_min(1)


class GRPOAdvantageEstimator:
    def __init__(self, cfg: dict, loss_cfg: Optional[dict] = None):
        self.use_leave_one_out_baseline = bool(cfg.get("use_leave_one_out_baseline", True))
        self.normalize_rewards = bool(cfg.get("normalize_rewards", True))

    def compute_advantage(self, prompt_ids, rewards, mask, valid_mask=None, **kwargs) -> torch.Tensor:
        valid = torch.ones_like(rewards) if valid_mask is None else valid_mask.to(rewards.dtype)
        base, std, trivial = calculate_baseline_and_std_per_prompt(
            prompt_ids, rewards, valid, leave_one_out_baseline=self.use_leave_one_out_baseline
        )
        adv = rewards - base
        if self.normalize_rewards:
            scale = (std > 0) & ~trivial
            adv = torch.where(scale, adv / (std + 1e-6), adv)
        return adv.unsqueeze(-1).expand(mask.shape)


def reward_component_keys(batch) -> list[str]:
    return sorted(k for k in batch.keys() if isinstance(k, str) and k.startswith("reward/"))


class GDPOAdvantageEstimator:
    def __init__(self, cfg: dict, loss_cfg: Optional[dict] = None):
        self.use_leave_one_out_baseline = bool(cfg.get("use_leave_one_out_baseline", True))
        self.normalize_rewards = bool(cfg.get("normalize_rewards", True))
        self.reward_weights = cfg.get("reward_weights")

    def compute_advantage(self, prompt_ids, rewards, mask, repeated_batch=None, valid_mask=None, **kwargs):
        keys = reward_component_keys(repeated_batch or {})
        if len(keys) < 2:
            raise ValueError(
                f"GDPO needs at least two reward components (reward/<name> keys); got {keys}. "
                "Use the 'grpo' estimator for a single reward."
            )
        weights = self.reward_weights or [1.0] * len(keys)
        if len(weights) != len(keys):
            raise ValueError(f"reward_weights has {len(weights)} entries for {len(keys)} components {keys}")
        ref = repeated_batch[keys[0]]
        valid = torch.ones_like(ref) if valid_mask is None else valid_mask.to(ref.dtype)
        total = torch.zeros_like(ref)
        for w, k in zip(weights, keys):
            r = repeated_batch[k].to(ref.dtype)
            base, std, trivial = calculate_baseline_and_std_per_prompt(
                prompt_ids, r, valid, leave_one_out_baseline=self.use_leave_one_out_baseline
            )
            a = r - base
            if self.normalize_rewards:
                a = torch.where((std > 0) & ~trivial, a / (std + 1e-6), a)
            total = total + w * a
        if valid.sum() <= 1:
            return torch.zeros_like(total).unsqueeze(-1).expand(mask.shape)
        mean = (total * valid).sum() / valid.sum()
        std = _masked_var(total, valid, mean).sqrt()
        total = total - mean
        if std > 0:
            total = total / std
        return total.unsqueeze(-1).expand(mask.shape)


class ReinforcePlusPlusAdvantageEstimator:
    def __init__(self, cfg: dict, loss_cfg: Optional[dict] = None):
        loss_cfg = loss_cfg or {}
        self.minus_baseline = bool(cfg.get("minus_baseline", True))
        self.use_kl_in_reward = bool(loss_cfg.get("use_kl_in_reward", False))
        self.kl_coef = float(loss_cfg.get("reference_policy_kl_penalty", 0.0))
        self.kl_type = loss_cfg.get("reference_policy_kl_type", "k3")

    def compute_advantage(self, prompt_ids, rewards, mask, logprobs_policy=None, logprobs_reference=None,
                          valid_mask=None, normalization_mask=None, **kwargs):
        if self.minus_baseline:
            valid = torch.ones_like(rewards) if valid_mask is None else valid_mask.to(rewards.dtype)
            mean, _, _ = calculate_baseline_and_std_per_prompt(prompt_ids, rewards, valid, leave_one_out_baseline=False)
            adv = rewards - mean
        else:
            adv = rewards
        adv = adv.unsqueeze(-1).expand(mask.shape)
        if self.use_kl_in_reward and logprobs_policy is not None and logprobs_reference is not None:
            kl = calculate_kl(logprobs_policy, logprobs_reference, kl_type=self.kl_type)
            kl = torch.where(torch.isneginf(logprobs_policy), torch.zeros_like(kl), kl)
            adv = adv - self.kl_coef * kl
        stats = mask if normalization_mask is None else normalization_mask
        n = stats.sum()
        if n == 0:
            return torch.zeros_like(adv)
        m = (adv * stats).sum() / n
        var = ((adv - m) ** 2 * stats).sum() / n
        return (adv - m) * var.clamp_min(1e-8).rsqrt()


class RawRewardAdvantageEstimator:
    def __init__(self, cfg: dict, loss_cfg: Optional[dict] = None):
        self.normalize_advantages = bool(cfg.get("normalize_advantages", True))

    def compute_advantage(self, prompt_ids, rewards, mask, **kwargs):
        adv = rewards.unsqueeze(-1).expand(mask.shape).to(torch.float32)
        if self.normalize_advantages:
            n = mask.sum().clamp_min(1)
            m = (adv * mask).sum() / n
            var = ((adv - m) ** 2 * mask).sum() / n
            adv = (adv - m) * var.clamp_min(1e-8).rsqrt()
        return adv, None


class GeneralizedAdvantageEstimator:
    """GAE for PPO with a critic.  ``values`` is ``[B, S]`` aligned with tokens."""

    def __init__(self, cfg: dict, loss_cfg: Optional[dict] = None):
        loss_cfg = loss_cfg or {}
        self.gae_lambda = float(cfg.get("gae_lambda", 0.95))
        self.gae_gamma = float(cfg.get("gae_gamma", 1.0))
        self.normalize_advantages = bool(cfg.get("normalize_advantages", True))
        self.gae_lambda_value = cfg.get("gae_lambda_value")
        self.gae_lambda_policy = cfg.get("gae_lambda_policy")
        self.length_adaptive_alpha = float(cfg.get("length_adaptive_alpha", 0.0))
        self.use_kl_in_reward = bool(loss_cfg.get("use_kl_in_reward", False))
        self.kl_coef = float(loss_cfg.get("reference_policy_kl_penalty", 0.0))
        self.kl_type = loss_cfg.get("reference_policy_kl_type", "k3")

    def token_level_rewards(self, rewards, mask, logprobs_policy=None, logprobs_reference=None):
        """Terminal reward at each row's last valid token, minus the KL penalty if enabled."""
        tok = torch.zeros_like(mask, dtype=torch.float32)
        if self.use_kl_in_reward and logprobs_policy is not None and logprobs_reference is not None:
            kl = calculate_kl(logprobs_policy, logprobs_reference, kl_type=self.kl_type)
            tok = tok - self.kl_coef * kl * mask
        S = mask.shape[1]
        pos = torch.arange(S, device=mask.device).expand_as(mask)
        last = torch.where(mask.bool(), pos, torch.full_like(pos, -1)).amax(-1)
        has = last >= 0
        rows = torch.arange(mask.shape[0], device=mask.device)[has]
        tok[rows, last[has]] += rewards[has].to(tok.dtype)
        return tok

    @staticmethod
    def gae(token_rewards, values, mask, gamma: float, lam) -> tuple[torch.Tensor, torch.Tensor]:
        """Backward recursion with carry-forward over masked positions.

        ``lam`` is a float or a per-row ``[B]`` tensor.  Returns (advantages, returns)."""
        B, S = token_rewards.shape
        adv = torch.zeros_like(token_rewards)
        last_gae = torch.zeros(B, dtype=token_rewards.dtype, device=token_rewards.device)
        next_v = torch.zeros_like(last_gae)
        lam_t = lam if isinstance(lam, torch.Tensor) else torch.full_like(last_gae, float(lam))
        for t in range(S - 1, -1, -1):
            m = mask[:, t].to(token_rewards.dtype)
            delta = token_rewards[:, t] + gamma * next_v - values[:, t]
            cand = delta + gamma * lam_t * last_gae
            last_gae = m * cand + (1 - m) * last_gae
            next_v = m * values[:, t] + (1 - m) * next_v
            adv[:, t] = cand * m
        returns = adv + values * mask
        return adv, returns

    def compute_advantage(self, prompt_ids, rewards, mask, values=None, logprobs_policy=None,
                          logprobs_reference=None, **kwargs):
        if values is None:
            raise ValueError("GAE needs per-token values from the critic")
        mask = mask.to(torch.float32)
        values = values.to(torch.float32)
        tok_r = self.token_level_rewards(rewards, mask, logprobs_policy, logprobs_reference)
        lam_pol = self.gae_lambda if self.gae_lambda_policy is None else self.gae_lambda_policy
        if self.length_adaptive_alpha > 0:
            lengths = mask.sum(-1).clamp_min(1)
            lam_pol = 1.0 - 1.0 / (self.length_adaptive_alpha * lengths)
        adv, _ = self.gae(tok_r, values, mask, self.gae_gamma, lam_pol)
        lam_val = self.gae_lambda if self.gae_lambda_value is None else self.gae_lambda_value
        _, returns = self.gae(tok_r, values, mask, self.gae_gamma, lam_val)
        if self.normalize_advantages:
            n = mask.sum().clamp_min(1)
            m = (adv * mask).sum() / n
            var = ((adv - m) ** 2 * mask).sum() / n
            adv = (adv - m) * var.clamp_min(1e-8).rsqrt() * mask
        return adv, returns


class OPDAdvantageEstimator:
    """On-policy distillation: ``A_t = log(alpha p_teacher + (1 - alpha) p_student) - log p_student``
    (plain OPD ``log p_teacher - log p_student`` at ``alpha = 1``; the trust-region
    mixture bounds the advantage below by ``log(1 - alpha)``), optionally centred
    by its mean over the valid tokens.  Reference: ``OPDAdvantageEstimator``
    (``nemo_rl/algorithms/advantage_estimator.py``)."""

    def __init__(self, cfg: dict, loss_cfg: Optional[dict] = None):
        self.alpha = float(cfg.get("proximal_teacher_alpha", 1.0))
        if not 0.0 < self.alpha <= 1.0:
            raise ValueError(f"proximal_teacher_alpha must be in (0, 1], got {self.alpha}")
        self.subtract_global_baseline = bool(cfg.get("subtract_global_baseline", False))
        self.last_metrics: dict = {}

    def compute_advantage(self, prompt_ids, rewards, mask, logprobs_policy=None, logprobs_teacher=None, **kwargs):
        # the reference's keyword names are accepted as well
        logprobs_teacher = kwargs.get("teacher_logprobs", logprobs_teacher)
        logprobs_policy = kwargs.get("prev_logprobs", logprobs_policy)
        if logprobs_policy is None or logprobs_teacher is None:
            raise ValueError("OPD needs student and teacher log-probabilities")
        m = mask.to(logprobs_policy.dtype)
        valid = m.bool()
        zero = torch.zeros_like(logprobs_policy)
        t = torch.where(valid, logprobs_teacher, zero)
        p = torch.where(valid, logprobs_policy, zero)
        gap = t - p
        if self.alpha >= 1.0:
            adv = gap
        else:
            adv = torch.logaddexp(t + math.log(self.alpha), p + math.log1p(-self.alpha)) - p
        adv = adv * m
        n = m.sum()
        if self.subtract_global_baseline and n > 0:
            adv = (adv - (adv * m).sum() / n) * m
        denom = n.clamp_min(1)
        mean = (adv * m).sum() / denom
        std = torch.sqrt((((adv - mean) * m) ** 2).sum() / denom)
        self.last_metrics = {
            "on_policy_distillation/adv_mean": float(mean),
            "on_policy_distillation/adv_std": float(std),
            "on_policy_distillation/teacher_student_logprob_gap_mean": float((gap * m).sum() / denom),
        }
        return adv


def make_advantage_estimator(cfg: dict, loss_cfg: Optional[dict] = None):
    name = (cfg or {}).get("name", "grpo")
    table = {
        "grpo": GRPOAdvantageEstimator,
        "gdpo": GDPOAdvantageEstimator,
        "reinforce_plus_plus": ReinforcePlusPlusAdvantageEstimator,
        "raw_reward": RawRewardAdvantageEstimator,
        "gae": GeneralizedAdvantageEstimator,
        "opd": OPDAdvantageEstimator,
    }
    if name not in table:
        raise ValueError(f"unknown advantage estimator {name!r}")
    return table[name](cfg or {}, loss_cfg or {})
