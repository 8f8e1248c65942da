"""RL / SFT / preference losses over sampled-token log-probabilities.

Reference semantics:
* ``ClippedPGLossFn`` - ``nemo_rl/algorithms/loss/loss_functions.py:173`` (config) and
  ``:698`` (``__call__``), objective in ``loss/clipped_pg.py:131``: PPO/GRPO clipped
  surrogate with asymmetric (clip-higher) bounds, dual clip, CISPO, GSPO
  sequence-level ratios, REINFORCE mode, forced on-policy ratio, reference KL
  (k1/k2/k3 with clamps, optional on-policy KL approximation), off-policy
  importance-sampling correction with TIS / ICE-POP / adaptive-PPO-clip /
  seq-mask-TIS truncation, VAPO positive-sample NLL and the diagnostic metrics
  (``probs_ratio*``, ``gen_kl_error``, ``policy_kl_error``,
  ``js_divergence_error``, ``approx_entropy``).
* ``NLLLossFn`` (``:1425``), ``DPOLossFn`` (``:1650``), ``PreferenceLossFn`` (reward
  model Bradley-Terry), ``DistillationLossFn``, ``ValueLossFn`` (clipped critic MSE
  for PPO).

Conventions (same as the reference): tensors are ``[B, S]`` aligned with input
tokens; the log-probability of token ``i`` sits at index ``i`` and position 0
carries 0.  ``next_token_logprobs`` is ``[B, S-1]`` = log p(token_{i+1} | <= i),
i.e. the data tensors sliced ``[:, 1:]``.  Losses are normalised by the GLOBAL
valid token (or sequence) count so that micro-batch and data-parallel partial
losses add up to the full-batch mean.
"""

from __future__ import annotations

from typing import Any, Optional

import torch
import torch.nn.functional as F

from rl_b200.algorithms.loss.interfaces import LossInputType, LossType
from rl_b200.algorithms.utils import calculate_kl, compute_seq_logprob_errors, masked_mean

__all__ = [
    "ClippedPGLossFn",
    "NLLLossFn",
    "DPOLossFn",
    "PreferenceLossFn",
    "DistillationLossFn",
    "ValueLossFn",
    "DEFAULT_CLIPPED_PG_CONFIG",
]

DEFAULT_CLIPPED_PG_CONFIG: dict[str, Any] = {
    "reference_policy_kl_penalty": 0.0,
    "reference_policy_kl_type": "k3",
    "kl_input_clamp_value": 20.0,
    "kl_output_clamp_value": 10.0,
    "ratio_clip_min": 0.2,
    "ratio_clip_max": 0.2,
    "ratio_clip_c": None,
    "use_on_policy_kl_approximation": False,
    "use_importance_sampling_correction": False,
    "truncated_importance_sampling_type": None,
    "truncated_importance_sampling_ratio": None,
    "truncated_importance_sampling_ratio_min": None,
    "truncated_importance_sampling_adaptive_target_entropy": 0.3,
    "truncated_importance_sampling_adaptive_k_step": 0.25,
    "truncated_importance_sampling_adaptive_k_max": 1.0,
    "truncated_importance_sampling_adaptive_outer_bound": 50.0,
    "sequence_level_importance_ratios": False,
    "token_level_loss": True,
    "force_on_policy_ratio": False,
    "seq_logprob_error_in_loss": False,
    "seq_logprob_error_threshold": None,
    "use_kl_in_reward": False,
    "use_cispo": False,
    "disable_ppo_ratio": False,
    "positive_example_nll_weight": 0.0,
    "score_centering": False,
    "metrics_level": "full",
}


def _m(x):
    """Metric value: kept on the device (detached) so that a training step reads all
    metrics back in one transfer instead of synchronising per micro-batch."""
    return x.detach() if isinstance(x, torch.Tensor) else float(x)


def _finite(x: torch.Tensor) -> torch.Tensor:
    return torch.nan_to_num(x, nan=0.0, posinf=0.0, neginf=0.0)


class ClippedPGLossFn:
    """Clipped policy-gradient loss for GRPO / PPO / DAPO / GSPO / CISPO."""

    input_type = LossInputType.LOGPROB

    def __init__(self, cfg: Optional[dict] = None):
        c = dict(DEFAULT_CLIPPED_PG_CONFIG)
        c.update({k: v for k, v in (cfg or {}).items() if v is not None or k in c})
        self.cfg = c
        self.kl_coef = float(c["reference_policy_kl_penalty"] or 0.0)
        self.kl_type = c["reference_policy_kl_type"]
        self.kl_in_clamp = c["kl_input_clamp_value"]
        self.kl_out_clamp = c["kl_output_clamp_value"]
        self.clip_lo = float(c["ratio_clip_min"])
        self.clip_hi = float(c["ratio_clip_max"])
        self.clip_c = float(c["ratio_clip_c"]) if c["ratio_clip_c"] is not None else -1.0
        if self.clip_c != -1.0 and self.clip_c <= 1.0:
            raise ValueError("ratio_clip_c (dual clip) must be > 1")
        self.on_policy_kl = bool(c["use_on_policy_kl_approximation"])
        self.use_is = bool(c["use_importance_sampling_correction"])
        self.tis_type = c["truncated_importance_sampling_type"]
        self.tis_max = c["truncated_importance_sampling_ratio"]
        self.tis_min = c["truncated_importance_sampling_ratio_min"]
        self.adaptive_k = 0.0
        self.seq_ratios = bool(c["sequence_level_importance_ratios"])
        self.token_level = bool(c["token_level_loss"])
        self.force_on_policy = bool(c["force_on_policy_ratio"])
        self.seq_err_in_loss = bool(c["seq_logprob_error_in_loss"])
        self.seq_err_threshold = c["seq_logprob_error_threshold"]
        self.use_cispo = bool(c["use_cispo"])
        self.disable_ratio = bool(c["disable_ppo_ratio"])
        self.nll_weight = float(c["positive_example_nll_weight"] or 0.0)
        # score centering: needs the sampler's top-k log-probs (rollout) and the
        # trainer's log-probs at those ids ("policy_logprobs_at_sampler_topk")
        self.score_centering = bool(c["score_centering"])
        if self.score_centering and (self.seq_ratios or (
                self.use_is and self.tis_type not in (None, "tis", "icepop"))):
            raise ValueError("score_centering composes with importance sampling off, untruncated token-level "
                             "IS, 'tis' or 'icepop'")
        self._sc_mode = (self.tis_type or "is") if self.use_is else "off"
        self.full_metrics = c["metrics_level"] == "full"
        self.loss_type = LossType.TOKEN_LEVEL if self.token_level else LossType.SEQUENCE_LEVEL
        if self.seq_ratios and self.token_level:
            # GSPO is defined with sequence-level normalisation.
            self.loss_type = LossType.SEQUENCE_LEVEL
            self.token_level = False
        if self.seq_err_in_loss and self.seq_err_threshold is None:
            raise ValueError("seq_logprob_error_in_loss needs seq_logprob_error_threshold")

    # -- adaptive-ppo-clip state (updated by the trainer between steps) --
    def update_adaptive_k(self, approx_entropy: float) -> None:
        c = self.cfg
        step = float(c["truncated_importance_sampling_adaptive_k_step"])
        kmax = float(c["truncated_importance_sampling_adaptive_k_max"])
        if approx_entropy < float(c["truncated_importance_sampling_adaptive_target_entropy"]):
            self.adaptive_k = min(kmax, self.adaptive_k + step)
        else:
            self.adaptive_k = max(0.0, self.adaptive_k - step)

    def _reduce(self, values, token_mask, sample_mask, mask, gtoks, gseqs):
        if self.token_level:
            return masked_mean(values, mask, global_normalization_factor=gtoks)
        per_seq = masked_mean(values, token_mask, dim=-1)
        return masked_mean(per_seq, sample_mask, global_normalization_factor=gseqs)

    def __call__(self, next_token_logprobs: torch.Tensor, data, global_valid_seqs: torch.Tensor,
                 global_valid_toks: torch.Tensor, **kwargs) -> tuple[torch.Tensor, dict]:
        curr = next_token_logprobs
        token_mask = data["token_mask"][:, 1:].to(curr.dtype)
        sample_mask = data["sample_mask"].to(curr.dtype)
        adv = data["advantages"][:, 1:].to(curr.dtype)
        gen_lp = data["generation_logprobs"][:, 1:].to(curr.dtype)
        prev_lp = curr.detach() if self.force_on_policy else data["prev_logprobs"][:, 1:].to(curr.dtype)

        # Rows without any loss token keep contributing to the global denominators
        # but nothing else.
        sample_mask = sample_mask * (token_mask > 0).any(-1).to(curr.dtype)
        mask = token_mask * sample_mask.unsqueeze(-1)
        metrics: dict[str, Any] = {}

        if self.seq_err_in_loss:
            errs, _ = compute_seq_logprob_errors(curr.detach(), gen_lp, token_mask, sample_mask)
            keep = (errs <= float(self.seq_err_threshold)).to(curr.dtype)
            metrics["num_masked_seqs_by_logprob_error"] = _m((sample_mask * (1 - keep)).sum())
            sample_mask = sample_mask * keep
            mask = token_mask * sample_mask.unsqueeze(-1)
            prev_lp = curr.detach()

        mb = mask.bool()
        zero = torch.zeros_like(curr)
        curr_m = torch.where(mb, curr, zero)
        prev_m = torch.where(mb, prev_lp, zero)
        gen_m = torch.where(mb, gen_lp, zero)

        # ---------------- reference-policy KL ----------------
        if self.kl_coef != 0.0:
            ref_lp = torch.where(mb, data["reference_policy_logprobs"][:, 1:].to(curr.dtype), zero)
            # with train-time top-k / top-p filtering the actor terms use the filtered
            # log-probs but the KL (and its weights) the unfiltered ones, consistent
            # with the unfiltered reference log-probs
            unf = data.get("curr_logprobs_unfiltered") if hasattr(data, "get") else None
            curr_kl = torch.where(mb, unf.to(curr.dtype), zero) if unf is not None else curr_m
            if self.on_policy_kl:
                w = torch.exp(curr_kl - gen_m)
            else:
                w = torch.exp(curr_kl - curr_kl.detach())
            w = _finite(w)
            kl_tok = self.kl_coef * calculate_kl(curr_kl, ref_lp, self.kl_type, self.kl_in_clamp,
                                                 self.kl_out_clamp, importance_sampling_weights=w)
            kl = self._reduce(kl_tok, token_mask, sample_mask, mask, global_valid_toks, global_valid_seqs)
        else:
            kl = curr.new_zeros(())

        # ---------------- off-policy IS weights ----------------
        is_w = None
        if self.use_is or self.full_metrics:
            if self.seq_ratios:
                is_w = _finite(torch.exp(((prev_m - gen_m) * mask).sum(-1))).detach().unsqueeze(-1)
            else:
                is_w = _finite(torch.exp(prev_m - gen_m)).detach()
            if self.tis_max is not None and self.tis_type is not None:
                is_w, oob = self._truncate_is(is_w, adv, prev_m, gen_m, mask)
                metrics["is_oob_ratio"] = oob

        # ---------------- actor objective ----------------
        if self.force_on_policy:
            ratios = torch.exp(curr_m - curr_m.detach())
            ratios_c = ratios
        elif not self.disable_ratio:
            log_r = curr_m - prev_m
            if self.seq_ratios:
                seq_lr = masked_mean(log_r, token_mask, dim=-1)
                ratios = torch.exp(seq_lr).unsqueeze(-1).expand_as(adv)
            else:
                ratios = torch.exp(log_r)
            ratios_c = ratios.clamp(1.0 - self.clip_lo, 1.0 + self.clip_hi)
        else:
            ratios = curr_m
            ratios_c = curr_m

        if self.use_cispo:
            per_tok = -adv * ratios_c.detach() * curr_m
        else:
            per_tok = torch.maximum(-adv * ratios, -adv * ratios_c)
        if self.clip_c > 0:
            per_tok = torch.where(adv < 0, torch.minimum(per_tok, -adv * self.clip_c), per_tok)
        if self.use_is and is_w is not None:
            per_tok = per_tok * is_w
        actor = self._reduce(per_tok, token_mask, sample_mask, mask, global_valid_toks, global_valid_seqs)
        if self.score_centering:
            from rl_b200.algorithms.loss.score_centering import score_centering_term

            plk = kwargs.get("policy_logprobs_at_sampler_topk")
            if plk is None and hasattr(data, "get"):
                plk = data.get("policy_logprobs_at_sampler_topk")
            if plk is None:
                raise ValueError("score_centering needs policy_logprobs_at_sampler_topk")
            bounds = None
            if self._sc_mode in ("tis", "icepop"):
                bounds = (float(self.tis_min or 0.0), float(self.tis_max))
            term, head = score_centering_term(plk, data["sampler_topk_logprobs"][:, 1:], self._sc_mode, bounds, mask)
            actor = actor + self._reduce(adv * term, token_mask, sample_mask, mask, global_valid_toks,
                                         global_valid_seqs)
            metrics["score_centering_head_mass"] = _m(masked_mean(head, mask,
                                                                  global_normalization_factor=global_valid_toks))

        loss = actor + kl
        if self.nll_weight > 0.0 and "rewards" in data:
            # VAPO: NLL on the tokens of correct samples (reward > 0), averaged over them
            correct = mask * (data["rewards"].to(curr.dtype) > 0).to(curr.dtype).unsqueeze(-1)
            n_ok = correct.sum()
            nll = torch.where(n_ok > 0, masked_mean(-curr_m, correct, global_normalization_factor=n_ok.clamp_min(1)),
                              curr.new_zeros(()))
            loss = loss + self.nll_weight * nll
            metrics["positive_nll"] = _m(nll.detach())

        with torch.no_grad():
            gtok = global_valid_toks
            metrics.update({
                "loss": _m(loss.detach()),
                "actor_loss": _m(actor.detach()),
                "kl_penalty": _m(kl.detach()),
                "num_valid_samples": _m(sample_mask.sum()),
            })
            if self.full_metrics:
                big = torch.full_like(ratios, float("inf"))
                metrics.update({
                    "probs_ratio": _m(masked_mean(ratios.detach(), mask, global_normalization_factor=gtok)),
                    "probs_ratio_clamped": _m(masked_mean(ratios_c.detach(), mask, global_normalization_factor=gtok)),
                    "probs_ratio_min": _m(torch.where(mb, ratios.detach(), big).min()),
                    "probs_ratio_max": _m(torch.where(mb, ratios.detach(), -big).max()),
                    "probs_ratio_clamped_min": _m(torch.where(mb, ratios_c.detach(), big).min()),
                    "probs_ratio_clamped_max": _m(torch.where(mb, ratios_c.detach(), -big).max()),
                })
                metrics.update(self._diagnostics(curr_m.detach(), prev_m, gen_m, mask, gtok))
        return loss, metrics

    def _truncate_is(self, w, adv, prev_m, gen_m, mask):
        kind = self.tis_type
        hi = float(self.tis_max)
        lo = self.tis_min
        if kind == "tis":
            lo = 0.0 if lo is None else float(lo)
            oob = ((w > hi) | (w < lo)).to(w.dtype)
            w = w.clamp(lo, hi)
        elif kind == "icepop":
            keep = (w >= float(lo)) & (w <= hi)
            oob = (~keep).to(w.dtype)
            w = torch.where(keep, w, torch.zeros_like(w))
        elif kind == "adaptive-ppo-clip":
            upper = hi + self.adaptive_k
            outer = float(self.cfg["truncated_importance_sampling_adaptive_outer_bound"])
            keep = (w <= outer) & ((adv >= 0) | (w >= float(lo))) & ((adv <= 0) | (w <= upper))
            oob = (~keep).to(w.dtype)
            w = torch.where(keep, w, torch.zeros_like(w))
        elif kind == "seq-mask-tis":
            n = mask.sum(-1).clamp_min(1)
            geo = torch.exp(((prev_m - gen_m) * mask).sum(-1) / n)
            keep = ((geo >= float(lo)) & (geo <= hi)).to(w.dtype)
            raw = _finite(torch.exp(prev_m - gen_m)).detach()
            w = raw * keep.unsqueeze(-1)
            oob_frac = _m(((1 - keep) * (mask.sum(-1) > 0).to(w.dtype)).sum())
            return w, oob_frac
        else:
            raise ValueError(f"unknown truncated_importance_sampling_type {kind!r}")
        return w, _m((oob.expand_as(mask) * mask).sum() / mask.sum().clamp_min(1))

    @staticmethod
    @torch.no_grad()
    def _diagnostics(curr_m, prev_m, gen_m, mask, gtok) -> dict:
        kl_gen = masked_mean(calculate_kl(gen_m, prev_m, "k3", None, None), mask, global_normalization_factor=gtok)
        kl_pol = masked_mean(calculate_kl(prev_m, gen_m, "k3", None, None), mask, global_normalization_factor=gtok)
        log_mix = torch.logaddexp(prev_m, gen_m) - torch.log(torch.tensor(2.0, dtype=prev_m.dtype, device=prev_m.device))
        a = prev_m - log_mix
        b = gen_m - log_mix
        js = masked_mean(0.5 * (torch.expm1(a) - a) + 0.5 * (torch.expm1(b) - b), mask, global_normalization_factor=gtok)
        ent = -masked_mean(torch.exp(curr_m - gen_m) * curr_m, mask, global_normalization_factor=gtok)
        mult_err = masked_mean(torch.exp((gen_m - prev_m).abs()), mask, global_normalization_factor=gtok)
        return {
            "gen_kl_error": _m(kl_gen),
            "policy_kl_error": _m(kl_pol),
            "js_divergence_error": _m(js),
            "approx_entropy": _m(ent),
            "token_mult_prob_error": _m(mult_err),
        }


class NLLLossFn:
    """Masked negative log-likelihood for SFT (token-level, globally normalised)."""

    input_type = LossInputType.LOGPROB
    loss_type = LossType.TOKEN_LEVEL

    def __call__(self, next_token_logprobs, data, global_valid_seqs, global_valid_toks, **kwargs):
        token_mask = data["token_mask"][:, 1:].to(next_token_logprobs.dtype)
        sample_mask = data["sample_mask"].to(next_token_logprobs.dtype)
        mask = token_mask * sample_mask.unsqueeze(-1)
        loss = masked_mean(-next_token_logprobs, mask, global_normalization_factor=global_valid_toks)
        return loss, {"loss": _m(loss.detach()), "num_unmasked_tokens": _m(mask.sum())}


def _seq_logprob(lp: torch.Tensor, mask: torch.Tensor, average: bool) -> torch.Tensor:
    s = (lp * mask).sum(-1)
    return s / mask.sum(-1).clamp_min(1) if average else s


class DPOLossFn:
    """Direct preference optimisation (sigmoid loss) + optional SFT term.

    Rows come in (chosen, rejected) pairs: even rows chosen, odd rows rejected
    (the reference's preference collate layout).
    """

    input_type = LossInputType.LOGPROB
    loss_type = LossType.SEQUENCE_LEVEL

    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        self.beta = float(cfg.get("reference_policy_kl_penalty", cfg.get("beta", 0.05)))
        self.preference_loss_weight = float(cfg.get("preference_loss_weight", 1.0))
        self.sft_loss_weight = float(cfg.get("sft_loss_weight", 0.0))
        self.average_log_probs = bool(cfg.get("preference_average_log_probs", False))
        self.sft_average_log_probs = bool(cfg.get("sft_average_log_probs", self.average_log_probs))

    def __call__(self, next_token_logprobs, data, global_valid_seqs, global_valid_toks, **kwargs):
        mask = data["token_mask"][:, 1:].to(next_token_logprobs.dtype) * data["sample_mask"].unsqueeze(-1)
        ref = data["reference_policy_logprobs"][:, 1:].to(next_token_logprobs.dtype)
        diff = _seq_logprob(next_token_logprobs - ref, mask, self.average_log_probs)
        chosen, rejected = diff[0::2], diff[1::2]
        margin = self.beta * (chosen - rejected)
        pair_mask = data["sample_mask"][0::2].to(margin.dtype)
        n_pairs = global_valid_seqs / 2
        pref = masked_mean(-F.logsigmoid(margin), pair_mask, global_normalization_factor=n_pairs)
        loss = self.preference_loss_weight * pref
        if self.sft_loss_weight > 0:
            chosen_lp = _seq_logprob(next_token_logprobs[0::2], mask[0::2], self.sft_average_log_probs)
            sft = masked_mean(-chosen_lp, pair_mask, global_normalization_factor=n_pairs)
            loss = loss + self.sft_loss_weight * sft
        acc = masked_mean((margin > 0).to(margin.dtype), pair_mask, global_normalization_factor=n_pairs)
        return loss, {
            "loss": _m(loss.detach()),
            "preference_loss": _m(pref.detach()),
            "accuracy": _m(acc),
            "rewards_chosen_mean": _m((self.beta * chosen).mean().detach()),
            "rewards_rejected_mean": _m((self.beta * rejected).mean().detach()),
        }


class MPOLossFn(DPOLossFn):
    """Mixed preference optimisation: DPO preference term + chosen-response SFT
    term + BCO quality term ``-log sigma(r_c - delta) - log sigma(-(r_r - delta))``
    with ``r = beta * log(pi / pi_ref)`` per sequence and a reward shift ``delta``
    kept as an EMA of the mean reward.

    Reference: ``MPOLossFn`` (``nemo_rl/algorithms/loss/loss_functions.py:1821``).  As
    there, the loss never mutates ``reward_shift`` itself: it reports
    ``bco_reward_sum`` / ``bco_reward_count`` (summed over micro-batches and DP),
    and the training loop calls ``update_reward_shift`` once per step, so every
    rank applies the same shift."""

    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        super().__init__(cfg)
        self.bco_loss_weight = float(cfg.get("bco_loss_weight", 1.0))
        self.quality_average_log_probs = bool(cfg.get("quality_average_log_probs", False))
        self.reward_shift_momentum = float(cfg.get("reward_shift_momentum", 0.9))
        self.reward_shift = float(cfg.get("reward_shift", 0.0))
        if not 0.0 <= self.reward_shift_momentum < 1.0:
            raise ValueError("reward_shift_momentum must be in [0, 1)")

    def update_reward_shift(self, reward_sum: float, reward_count: float) -> float:
        if reward_count > 0:
            m = self.reward_shift_momentum
            self.reward_shift = m * self.reward_shift + (1.0 - m) * reward_sum / reward_count
        return self.reward_shift

    def __call__(self, next_token_logprobs, data, global_valid_seqs, global_valid_toks, **kwargs):
        loss, metrics = super().__call__(next_token_logprobs, data, global_valid_seqs, global_valid_toks)
        mask = data["token_mask"][:, 1:].to(next_token_logprobs.dtype) * data["sample_mask"].unsqueeze(-1)
        ref = data["reference_policy_logprobs"][:, 1:].to(next_token_logprobs.dtype)
        q = self.beta * _seq_logprob(next_token_logprobs - ref, mask, self.quality_average_log_probs)
        smask = data["sample_mask"].to(q.dtype)
        c_mask, r_mask = smask[0::2], smask[1::2]
        n_pairs = global_valid_seqs / 2
        delta = torch.as_tensor(self.reward_shift, dtype=q.dtype, device=q.device)
        bco = (masked_mean(-F.logsigmoid(q[0::2] - delta), c_mask, global_normalization_factor=n_pairs)
               + masked_mean(-F.logsigmoid(-(q[1::2] - delta)), r_mask, global_normalization_factor=n_pairs))
        loss = loss + self.bco_loss_weight * bco
        metrics.update({
            "loss": _m(loss.detach()),
            "bco_loss": _m(bco.detach()),
            "bco_reward_sum": _m((q.detach() * smask).sum()),
            "bco_reward_count": _m(smask.sum()),
        })
        return loss, metrics


class PreferenceLossFn:
    """Bradley-Terry reward-model loss over scalar rewards of (chosen, rejected) pairs."""

    input_type = LossInputType.VALUE
    loss_type = LossType.SEQUENCE_LEVEL

    def __call__(self, rewards: torch.Tensor, data, global_valid_seqs, global_valid_toks, **kwargs):
        if rewards.dim() == 2:
            # per-token values: the sequence reward is the value at its last token
            last = (data["input_lengths"].to(rewards.device).long() - 1).clamp_min(0)
            rewards = rewards.gather(1, last.unsqueeze(1)).squeeze(1)
        chosen, rejected = rewards[0::2], rewards[1::2]
        pair_mask = data["sample_mask"][0::2].to(rewards.dtype)
        n_pairs = global_valid_seqs / 2
        loss = masked_mean(-F.logsigmoid(chosen - rejected), pair_mask, global_normalization_factor=n_pairs)
        acc = masked_mean((chosen > rejected).to(rewards.dtype), pair_mask, global_normalization_factor=n_pairs)
        return loss, {"loss": _m(loss.detach()), "accuracy": _m(acc)}


class DistillationLossFn:
    """Token-level KL between student and teacher top-k distributions.

    ``student_logits`` ``[B, S-1, V]`` (or top-k gathered), teacher top-k
    log-probs / indices in ``data['teacher_topk_logprobs']`` and
    ``data['teacher_topk_indices']``.  ``kl_type``: forward / reverse / mixed.
    """

    input_type = LossInputType.LOGIT
    loss_type = LossType.TOKEN_LEVEL

    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        self.kl_type = cfg.get("kl_type", "forward")
        self.mixed_kl_weight = float(cfg.get("mixed_kl_weight", 0.5))
        self.zero_outside_topk = bool(cfg.get("zero_outside_topk", False))

    def __call__(self, student_logits, data, global_valid_seqs, global_valid_toks, **kwargs):
        mask = data["token_mask"][:, 1:].to(torch.float32) * data["sample_mask"].unsqueeze(-1)
        s_logp_full = torch.log_softmax(student_logits.float(), dim=-1)
        idx = data["teacher_topk_indices"][:, 1:]
        t_logp = data["teacher_topk_logprobs"][:, 1:].float()
        s_logp = torch.gather(s_logp_full, -1, idx.long())
        if self.zero_outside_topk:
            s_logp = s_logp - torch.logsumexp(s_logp, -1, keepdim=True)
            t_logp = t_logp - torch.logsumexp(t_logp, -1, keepdim=True)
        t_p, s_p = t_logp.exp(), s_logp.exp()
        fwd = (t_p * (t_logp - s_logp)).sum(-1)
        rev = (s_p * (s_logp - t_logp)).sum(-1)
        if self.kl_type == "forward":
            tok = fwd
        elif self.kl_type == "reverse":
            tok = rev
        else:
            tok = self.mixed_kl_weight * fwd + (1 - self.mixed_kl_weight) * rev
        loss = masked_mean(tok, mask, global_normalization_factor=global_valid_toks)
        return loss, {"loss": _m(loss.detach())}


class ValueLossFn:
    """Clipped value loss for the PPO critic: max((V-R)^2, (clip(V)-R)^2) / 2."""

    input_type = LossInputType.VALUE
    loss_type = LossType.TOKEN_LEVEL

    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        self.clip = cfg.get("value_clip", 0.2)

    def __call__(self, values, data, global_valid_seqs, global_valid_toks, **kwargs):
        mask = data["token_mask"].to(values.dtype) * data["sample_mask"].unsqueeze(-1)
        returns = data["returns"].to(values.dtype)
        old = data["old_values"].to(values.dtype)
        l1 = (values - returns) ** 2
        if self.clip is not None:
            vc = old + (values - old).clamp(-float(self.clip), float(self.clip))
            l1 = torch.maximum(l1, (vc - returns) ** 2)
        loss = 0.5 * masked_mean(l1, mask, global_normalization_factor=global_valid_toks)
        return loss, {"value_loss": _m(loss.detach())}
