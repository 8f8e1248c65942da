"""Asynchronous GRPO training loop.

Reference: ``async_grpo_train`` (``nemo_rl/algorithms/grpo.py:5257``) with the
replay buffer / trajectory collector of ``nemo_rl/algorithms/async_utils``.
Config keys (``grpo.async_grpo``): ``enabled``, ``max_trajectory_age_steps``,
``in_flight_weight_updates``, ``max_generation_failures``; the loss should
enable ``use_importance_sampling_correction`` because trajectories may come
from weights up to ``max_trajectory_age_steps`` updates old.

One rank = one trainer + one rollout pump thread (``AsyncTrajectoryCollector``).
The trainer takes, at weight version ``v``, the groups generated for step
``v``; it computes advantages, the current policy's logprobs (``prev_logprobs``,
so the clipped ratio is against the current weights, with the rollout
logprobs kept for the importance-sampling correction), trains one step through
the split train API and bumps the version the pump generates with.

Rollout generation in the pump thread issues no collectives: tensor-parallel
generation (collectives on the TP group from two threads) is not supported in
async mode, so the policy must be TP=1 for generation.
"""

from __future__ import annotations

import os

import time
from typing import Optional

import torch

from rl_b200.algorithms.advantage_estimator import make_advantage_estimator
from rl_b200.algorithms.async_utils import AsyncTrajectoryCollector, ReplayBuffer, groups_to_batch, wait_for_groups
from rl_b200.algorithms.grpo import DEFAULT_GRPO_CONFIG, GRPOSaveState, _dp_sum, build_train_data, validate
from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
from rl_b200.algorithms.utils import set_seed
from rl_b200.algorithms.length_penalty import LengthPenaltyConfig, apply_length_penalty_to_rollout
from rl_b200.experience.rollouts import run_multi_turn_rollout
from rl_b200.utils.timer import Timer, max_over_ranks

__all__ = ["async_grpo_train"]


def replay_buffer_file() -> str:
    """Per-rank replay-buffer file in a checkpoint directory (every rank keeps its own buffer)."""
    import torch.distributed as dist

    return f"replay_buffer_rank{dist.get_rank() if dist.is_initialized() else 0}.pt"


def rollout_recovery_file() -> str:
    """Per-rank rollout-recovery ledger file in a checkpoint directory."""
    import torch.distributed as dist

    return f"rollout_recovery_rank{dist.get_rank() if dist.is_initialized() else 0}.pt"


def restore_rollout_recovery(ckpt_dir: str):
    """This rank's rollout-recovery ledger from a checkpoint, or None when absent."""
    from rl_b200.experience.rollout_recovery import RolloutRecoveryLedger

    path = os.path.join(ckpt_dir, rollout_recovery_file())
    return RolloutRecoveryLedger.load(path) if os.path.exists(path) else None


def restore_replay_buffer(ckpt_dir: str, num_prompt_groups: int, max_size: int,
                          load_replay_buffer: Optional[bool] = None) -> Optional[ReplayBuffer]:
    """The checkpoint's replay buffer of this rank (groups of incomplete targets
    dropped), or None when disabled (``load_replay_buffer: false``) or absent.
    Reference: ``_maybe_restore_async_replay_buffer_checkpoint`` (``nemo_rl/algorithms/grpo.py``)."""
    import torch

    path = os.path.join(ckpt_dir, replay_buffer_file())
    if load_replay_buffer is False or not os.path.exists(path):
        return None
    buf = ReplayBuffer(max_size=max_size)
    buf.load_state_dict(torch.load(path, weights_only=False), drop_incomplete_targets=num_prompt_groups)
    return buf


def async_grpo_train(policy, dataloader, task_to_env: dict, master_config: dict, loss_fn=None, logger=None,
                     checkpointer=None, save_state: Optional[GRPOSaveState] = None, val_dataloader=None,
                     val_task_to_env: Optional[dict] = None, tokenizer=None, max_steps: Optional[int] = None,
                     step_callback=None, replay_buffer: Optional[ReplayBuffer] = None,
                     wait_timeout_s: float = 3600.0, rollout_ledger=None) -> GRPOSaveState:
    """Async GRPO: a rollout pump thread fills a replay buffer while the trainer
    consumes groups generated at most ``max_trajectory_age_steps`` versions ago.
    ``rollout_ledger`` (restored from a checkpoint) makes the pump regenerate the
    prompt groups that were in flight when that checkpoint was written; the
    ledger of this run is saved with every checkpoint."""
    from rl_b200.experience.rollout_recovery import RolloutRecoveryLedger

    ps = policy.ps
    if ps.tp_size > 1:
        raise NotImplementedError("async GRPO generates in a side thread and needs TP=1 generation")
    cfg = {**DEFAULT_GRPO_CONFIG, **master_config.get("grpo", {})}
    acfg = {**DEFAULT_GRPO_CONFIG["async_grpo"], **(cfg.get("async_grpo") or {})}
    if cfg.get("length_penalty") is not None:
        cfg["length_penalty"] = LengthPenaltyConfig(cfg["length_penalty"])
    max_age = int(acfg.get("max_trajectory_age_steps", 1))
    loss_cfg = master_config.get("loss_fn", {})
    loss_fn = loss_fn or ClippedPGLossFn(loss_cfg)
    adv_cfg = dict(cfg.get("adv_estimator", {}) or {})
    adv_cfg.setdefault("normalize_rewards", cfg["normalize_rewards"])
    adv_cfg.setdefault("use_leave_one_out_baseline", cfg["use_leave_one_out_baseline"])
    estimator = make_advantage_estimator(adv_cfg, loss_cfg)
    G = int(cfg["num_generations_per_prompt"])
    n_groups = max(1, int(cfg["num_prompts_per_step"]) // max(1, ps.dp_size))
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    kl_on = float(loss_cfg.get("reference_policy_kl_penalty", 0.0) or 0.0) != 0.0
    state = save_state or GRPOSaveState.default()
    step = int(state["current_step"])
    max_steps = max_steps if max_steps is not None else int(cfg["max_num_steps"])
    set_seed(int(cfg["seed"]) + ps.dp_rank)
    buffer = replay_buffer or ReplayBuffer(max_size=n_groups * (max_age + 1) * 2)
    engine = getattr(policy, "engine", None)
    if engine is not None:
        engine.capture_error_mode = "thread_local"
        # the KV cache may not borrow the gradient arena: training runs meanwhile
        engine.kv_arena = None

    def rollout_fn(batch, target):
        rep = batch.repeat_interleave(G)
        n_prompts = len(batch["message_log"])
        base = target * 1_000_000 + ps.dp_rank * n_prompts
        rep["group_id"] = torch.arange(base, base + n_prompts).repeat_interleave(G)
        policy.prepare_for_generation(len(rep["message_log"]))
        rollout, metrics = run_multi_turn_rollout(policy, rep, tokenizer, task_to_env, max_seq,
                                                  int(cfg["max_rollout_turns"]))
        if cfg.get("length_penalty") is not None:  # training rollouts only
            metrics.update(apply_length_penalty_to_rollout(rollout, cfg["length_penalty"], G, tokenizer))
        return rollout, metrics

    restart = []
    if rollout_ledger is not None:
        live = _buffer_group_ids(replay_buffer.state_dict()) if replay_buffer is not None else None
        restart = rollout_ledger.prepare_for_restart(live)
    ledger = rollout_ledger or RolloutRecoveryLedger()
    collector = AsyncTrajectoryCollector(rollout_fn, dataloader, buffer, n_groups, G, max_age,
                                         initial_weight_version=step,
                                         in_flight_weight_updates=bool(acfg.get("in_flight_weight_updates", False)),
                                         max_generation_failures=int(acfg.get("max_generation_failures", 0)),
                                         ledger=ledger, restart_groups=restart)
    collector.start()
    timer = Timer()
    try:
        while step < max_steps:
            timer.reset()
            t_step = time.perf_counter()
            with timer.time("total_step_time"):
                with timer.time("exposed_generation"):
                    try:
                        sample = wait_for_groups(buffer, collector, n_groups, step, max_age, wait_timeout_s)
                    except StopIteration:
                        break
                consumed = [g["recovery_group_id"][0] for g in sample["trajectories"] if "recovery_group_id" in g]
                ledger.mark_consumed([c for c in consumed if c in ledger])
                rollout = groups_to_batch(sample["trajectories"])
                with timer.time("data_processing"):
                    train_data, adv_stats = build_train_data(rollout, estimator, cfg, loss_cfg, rollout["group_id"])
                with timer.time("policy_and_reference_logprobs"):
                    policy.prepare_for_lp_inference()
                    train_data["prev_logprobs"] = policy.get_logprobs(train_data)["logprobs"]
                    if kl_on:
                        train_data["reference_policy_logprobs"] = \
                            policy.get_reference_policy_logprobs(train_data)["reference_logprobs"]
                with timer.time("policy_training"):
                    policy.prepare_for_training()
                    st = policy.begin_train_step(train_data, loss_fn)
                    for i in range(st.num_microbatches):
                        policy.train_microbatch(st, i)
                    # the update and the refit exclude rollouts that must not see a
                    # half-written model (in-flight updates only exclude the write)
                    with collector.weights_lock:
                        train_results = policy.finish_train_step(st)
                        with timer.time("weight_sync"):
                            policy.refit()
                step += 1
                collector.set_weight_version(step)
            step_time = time.perf_counter() - t_step
            tok = float(train_data["input_lengths"].sum())
            tok_all = _dp_sum(tok, ps) if ps.dp_size > 1 else tok
            step_time_max = max_over_ranks(step_time)
            metrics = dict(train_results)
            metrics.update(adv_stats)
            metrics.update(collector.efficiency_metrics())
            metrics.update({f"rollout_recovery/{k}": float(v) for k, v in ledger.counts().items()})
            metrics.update({"avg_trajectory_age": sample["avg_trajectory_age"], "buffer_size": buffer.size(),
                            "total_tokens": tok_all, "tokens_per_sec": tok_all / step_time_max,
                            "tokens_per_sec_per_gpu": tok_all / step_time_max / max(1, ps.world_size),
                            "step_time_s": step_time_max})
            timing = timer.get_timing_metrics()
            state["current_step"] = step
            state["total_steps"] = int(state.get("total_steps", 0)) + 1
            state["consumed_samples"] = int(state.get("consumed_samples", 0)) + n_groups * ps.dp_size
            if logger:
                logger.log_metrics(metrics, step, prefix="train")
                logger.log_metrics(timing, step, prefix="timing/train")
            if step_callback is not None:
                step_callback(step, {**metrics, **{"timing/" + k: v for k, v in timing.items()}})
            val_period = int(cfg.get("val_period") or 0)
            if val_dataloader is not None and val_period > 0 and step % val_period == 0:
                with collector.weights_lock:
                    vm = validate(policy, val_dataloader, val_task_to_env or task_to_env, master_config, step,
                                  tokenizer)
                if logger:
                    logger.log_metrics(vm, step, prefix="validation")
            if checkpointer is not None and checkpointer.should_save(step):
                with collector.weights_lock:
                    buf_sd = buffer.state_dict()
                    ledger.prune_sealed(_buffer_group_ids(buf_sd))
                    checkpointer.save(policy, state, dataloader, metrics, step,
                                      rank_files={replay_buffer_file(): buf_sd,
                                                  rollout_recovery_file(): ledger.state_dict()})
    finally:
        collector.stop()
    collector.check_health()
    return state


def _buffer_group_ids(buffer_state: dict) -> list[str]:
    """Ledger ids of the prompt groups held in a replay-buffer state dict."""
    return [g["recovery_group_id"][0] for g in buffer_state.get("groups", []) if "recovery_group_id" in g]
