"""PPO with a learned critic (reference: ``PPOConfig`` ``nemo_rl/algorithms/ppo.py:191``,
``ppo_train`` ``:1329``; value models ``nemo_rl/models/value/*``, GAE
``advantage_estimator.py:381``).

Per step: rollouts -> rewards -> critic values -> GAE advantages / returns ->
clipped-PG policy update -> clipped value-loss critic update -> refit.  The
critic is a policy worker built with a scalar value head (``num_labels: 1``);
V(s_t) for response token t is the critic's output at position t-1 (the state
that produced token t).
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.algorithms.advantage_estimator import GeneralizedAdvantageEstimator, RawRewardAdvantageEstimator
from rl_b200.algorithms.grpo import build_train_data
from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn, ValueLossFn
from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.experience.rollouts import run_multi_turn_rollout

__all__ = ["ppo_train", "token_values"]


def token_values(values: torch.Tensor) -> torch.Tensor:
    """Shift critic outputs so that column t holds V(state before token t)."""
    out = torch.zeros_like(values)
    out[:, 1:] = values[:, :-1]
    return out


class _PassThrough:
    """Estimator stub: build_train_data needs one; PPO replaces the advantages."""

    def compute_advantage(self, prompt_ids, rewards, mask, **kw):
        return torch.zeros_like(mask)


def ppo_train(policy, critic, dataloader, task_to_env: dict, master_config: dict, logger=None, checkpointer=None,
              save_state=None, max_steps: Optional[int] = None, step_callback=None, tokenizer=None) -> dict:
    cfg = master_config.get("ppo", {})
    loss_cfg = master_config.get("loss_fn", {})
    adv_cfg = cfg.get("adv_estimator", {"name": "gae"})
    est = GeneralizedAdvantageEstimator(adv_cfg, loss_cfg) if adv_cfg.get("name", "gae") == "gae" \
        else RawRewardAdvantageEstimator(adv_cfg, loss_cfg)
    pg_loss = ClippedPGLossFn(loss_cfg)
    v_loss = ValueLossFn(cfg.get("value_loss", {}))
    G = int(cfg.get("num_generations_per_prompt", 1))
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    max_steps = int(max_steps if max_steps is not None else cfg.get("max_num_steps", 10 ** 9))
    kl_on = float(loss_cfg.get("reference_policy_kl_penalty", 0.0) or 0.0) != 0.0
    state = dict(save_state or {"current_step": 0})
    step = int(state["current_step"])
    for batch in dataloader:
        if step >= max_steps:
            break
        rep = batch.repeat_interleave(G)
        n = len(batch["message_log"])
        rep["group_id"] = torch.arange(n).repeat_interleave(G)
        policy.prepare_for_generation(len(rep["message_log"]))
        rollout, rmetrics = run_multi_turn_rollout(policy, rep, tokenizer, task_to_env, max_seq,
                                                   int(cfg.get("max_rollout_turns", 1)))
        policy.finish_generation()
        data, stats = build_train_data(rollout, _PassThrough(), cfg, loss_cfg, rollout["group_id"])
        data["prev_logprobs"] = policy.get_logprobs(data)["logprobs"]
        if kl_on:
            data["reference_policy_logprobs"] = policy.get_reference_policy_logprobs(data)["reference_logprobs"]
        values = token_values(critic.get_values(data)["values"])
        rewards = rollout["total_reward"].float()
        mask = data["token_mask"]
        if isinstance(est, GeneralizedAdvantageEstimator):
            adv, returns = est.compute_advantage(rep["group_id"], rewards, mask, values=values,
                                                 logprobs_policy=data["prev_logprobs"],
                                                 logprobs_reference=data.get("reference_policy_logprobs"))
        else:
            adv, _ = est.compute_advantage(rep["group_id"], rewards, mask)
            returns = rewards.unsqueeze(-1).expand_as(mask) * mask
        data["advantages"] = adv * mask
        pres = policy.train(data, pg_loss)
        cdata = BatchedDataDict({"input_ids": data["input_ids"], "input_lengths": data["input_lengths"],
                                 "token_mask": mask, "sample_mask": data["sample_mask"],
                                 "returns": returns * mask, "old_values": values})
        # critic predicts V at position t-1 for token t: shift targets back by one
        for k in ("returns", "old_values", "token_mask"):
            t = cdata[k]
            s = torch.zeros_like(t)
            s[:, :-1] = t[:, 1:]
            cdata[k] = s
        cres = critic.train(cdata, v_loss)
        policy.refit()
        step += 1
        state["current_step"] = step
        metrics = {"loss": pres["loss"], "value_loss": cres.get("value_loss", cres["loss"]),
                   "reward_mean": float(rewards.mean()), "grad_norm": pres["grad_norm"],
                   "critic_grad_norm": cres["grad_norm"]}
        metrics.update({k: v for k, v in pres.items() if k.startswith(("probs_ratio", "gen_kl", "approx"))})
        if logger:
            logger.log_metrics(metrics, step, prefix="train")
        if step_callback:
            step_callback(step, metrics)
        if checkpointer is not None and checkpointer.should_save(step):
            checkpointer.save(policy, state, dataloader, metrics, step)
    return state
