"""GRPO / DAPO / GSPO training loop.

Reference: ``nemo_rl/algorithms/grpo.py`` - ``GRPOConfig`` ``:356``, ``GRPOSaveState``
``:439``, ``MasterConfig`` ``:542``, ``setup`` ``:667``, ``dynamic_sampling`` ``:2168``,
``scale_rewards`` ``:2312``, ``refit_policy_generation`` ``:3150``, ``_grpo_train_impl``
``:3574`` (step stages in section 3.2 of the survey), ``validate`` ``:4897``.

SPMD design: every rank runs this loop.  Each data-parallel rank draws its own
``num_prompts_per_step / dp`` prompts and generates ALL samples of those prompts,
so prompt groups never straddle ranks: rewards, baselines and advantages are
computed locally, and only scalars (valid-token counts, metrics, loss) cross
ranks.  Tensor-parallel peers draw identical prompts and sample identical
tokens (same seed; logits are all-gathered before sampling).
"""

from __future__ import annotations

import copy
import math
import os
import time
from typing import Any, Optional

import torch
import torch.distributed as dist

from rl_b200.algorithms.advantage_estimator import make_advantage_estimator
from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
from rl_b200.algorithms.utils import calculate_baseline_and_std_per_prompt, set_seed
from rl_b200.data.llm_message_utils import add_loss_mask_to_message_log, batched_message_log_to_flat_message
from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.algorithms.length_penalty import LengthPenaltyConfig, apply_length_penalty_to_rollout
from rl_b200.experience.rollouts import run_multi_turn_rollout
from rl_b200.utils.flops import FLOPTracker, mfu
from rl_b200.utils.nvtx import maybe_gpu_profile_step
from rl_b200.utils.timer import Timer, max_over_ranks

__all__ = ["DEFAULT_GRPO_CONFIG", "GRPOSaveState", "grpo_train", "build_train_data", "dynamic_sampling",
           "scale_rewards", "apply_reward_shaping", "validate", "refit_policy_generation"]

DEFAULT_GRPO_CONFIG: dict[str, Any] = {
    "num_prompts_per_step": 8,
    "num_generations_per_prompt": 4,
    "max_rollout_turns": 1,
    "max_num_epochs": 1,
    "max_num_steps": 1000000,
    "normalize_rewards": True,
    "use_leave_one_out_baseline": True,
    "val_period": 0,
    "val_at_start": False,
    "val_at_end": False,
    "max_val_samples": 256,
    "val_batch_size": 256,
    "val_num_generations_per_prompt": 1,
    "stop_at_validation_metric": None,
    "stop_at_validation_threshold": None,
    "seed": 42,
    "overlong_filtering": False,
    "advantage_clip_low": None,
    "advantage_clip_high": None,
    "use_dynamic_sampling": False,
    "dynamic_sampling_max_gen_batches": 10,
    "batch_multiplier": 1,
    "reward_shaping": {"enabled": False},
    "reward_scaling": {"enabled": False},
    "adv_estimator": {"name": "grpo"},
    "seq_logprob_error_threshold": None,
    "async_grpo": {"enabled": False, "max_trajectory_age_steps": 1},
}


class GRPOSaveState(dict):
    """Resumable loop state (reference ``GRPOSaveState`` ``grpo.py:439``)."""

    @classmethod
    def default(cls) -> "GRPOSaveState":
        return cls(current_step=0, current_epoch=0, total_steps=0, consumed_samples=0, total_valid_tokens=0,
                   val_reward=None)


def refit_policy_generation(policy) -> float:
    """Push trained weights to the rollout engine.  Colocated on one device with
    the same layout, the optimizer already wrote the bf16 weights the engine
    reads, so this only validates / re-quantises (fp8 rollout)."""
    return policy.refit()


def apply_reward_shaping(rewards: torch.Tensor, gen_lengths: torch.Tensor, cfg: dict,
                         truncated: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reward shaping.

    * DAPO overlong penalty (``overlong_buffer_length``, ``overlong_buffer_penalty``,
      ``max_response_length``): a response longer than ``max - buffer`` tokens loses
      ``(length - (max - buffer)) / buffer * penalty`` (linear, not capped);
    * ``stop_properly_penalty_coef`` in [0, 1]: truncated responses' rewards are
      multiplied by it.

    ``gen_lengths`` counts every generated assistant token of the sample.
    Reference: ``apply_reward_shaping`` (``nemo_rl/algorithms/reward_functions.py``)."""
    if not cfg or not cfg.get("enabled", False):
        return rewards
    out = rewards.clone()
    coef = cfg.get("stop_properly_penalty_coef")
    if coef is not None:
        coef = float(coef)
        assert 0.0 <= coef <= 1.0, f"stop_properly_penalty_coef must be in [0, 1], got {coef}"
        assert truncated is not None, "truncated field not found (needed by stop_properly_penalty_coef)"
        out = torch.where(truncated.to(torch.bool), out * coef, out)
    keys = ("overlong_buffer_length", "overlong_buffer_penalty", "max_response_length")
    if coef is None or any(cfg.get(k) is not None for k in keys):
        if any(cfg.get(k) is None for k in keys):
            raise ValueError("DAPO reward shaping is currently supported with overlong_buffer_length, "
                             "overlong_buffer_penalty and max_response_length all set")
        buf = float(cfg["overlong_buffer_length"])
        pen = float(cfg["overlong_buffer_penalty"])
        expected = float(cfg["max_response_length"]) - buf
        exceed = gen_lengths.to(out.dtype) - expected
        out = out + torch.clamp(-exceed / max(buf, 1e-12) * pen, max=0.0)
    return out


def scale_rewards(rewards: torch.Tensor, cfg: dict) -> torch.Tensor:
    """Linear map ``[source_min, source_max] -> [target_min, target_max]`` (clamped)."""
    if not cfg or not cfg.get("enabled", False):
        return rewards
    smin, smax = float(cfg.get("source_min", 0.0)), float(cfg.get("source_max", 1.0))
    tmin, tmax = float(cfg.get("target_min", 0.0)), float(cfg.get("target_max", 1.0))
    r = rewards.clamp(smin, smax)
    return tmin + (r - smin) * (tmax - tmin) / max(smax - smin, 1e-12)


def dynamic_sampling(rewards: torch.Tensor, group_ids: torch.Tensor,
                     valid: Optional[torch.Tensor] = None) -> torch.Tensor:
    """DAPO dynamic sampling: keep only rows of groups whose rewards are not all
    equal (a constant group has zero advantage everywhere), judged on the whole
    group (not leave-one-out peers), so a mixed group is kept entire.  ``valid``
    (masked_reward_policy "exclude") limits the vote to rows with a loss weight.
    Returns a row mask."""
    vm = torch.ones_like(rewards) if valid is None else valid.to(rewards.dtype)
    _, std, trivial = calculate_baseline_and_std_per_prompt(group_ids, rewards, vm, leave_one_out_baseline=False)
    return ~trivial


def apply_message_level_advantage_penalties(train_data: BatchedDataDict, message_logs: list,
                                            invalid_tool_call_advantage: Optional[float] = None,
                                            malformed_thinking_advantage: Optional[float] = None) -> None:
    """Overwrite the advantages of the tokens of assistant messages that an
    environment flagged (``is_invalid_tool_call`` / ``has_malformed_thinking``)
    with the configured values; other messages and tokens keep theirs.  A
    broadcast (stride-0) advantage tensor is materialised first.
    Reference: ``_apply_message_level_advantage_penalties`` (``nemo_rl/algorithms/grpo.py``)."""
    if invalid_tool_call_advantage is None and malformed_thinking_advantage is None:
        return
    adv = train_data["advantages"].clone()
    for b, log in enumerate(message_logs):
        off = 0
        for msg in log:
            L = len(msg["token_ids"])
            if msg.get("role") == "assistant":
                val = None
                if invalid_tool_call_advantage is not None and msg.get("is_invalid_tool_call"):
                    val = float(invalid_tool_call_advantage)
                elif malformed_thinking_advantage is not None and msg.get("has_malformed_thinking"):
                    val = float(malformed_thinking_advantage)
                if val is not None:
                    adv[b, off:off + L] = val
            off += L
    train_data["advantages"] = adv


def build_train_data(rollout_batch: BatchedDataDict, advantages_fn, cfg: dict, loss_cfg: dict,
                     group_ids: torch.Tensor) -> tuple[BatchedDataDict, dict]:
    """Flatten message logs and compute per-token advantages."""
    logs = rollout_batch["message_log"]
    add_loss_mask_to_message_log(logs, roles_to_train_on=("assistant",))
    flat, lengths = batched_message_log_to_flat_message(logs)
    token_mask = flat["token_loss_mask"].float()
    rewards = rollout_batch["total_reward"].float()
    gen_len = token_mask.sum(-1)
    rewards = apply_reward_shaping(rewards, gen_len, cfg.get("reward_shaping", {}),
                                   rollout_batch["truncated"] if "truncated" in rollout_batch else None)
    rewards = scale_rewards(rewards, cfg.get("reward_scaling", {}))
    sample_mask = rollout_batch["loss_multiplier"].float().clone()
    if cfg.get("overlong_filtering", False):
        sample_mask = sample_mask * (~rollout_batch["truncated"]).float()
    # masked_reward_policy "exclude": rows with zero loss weight do not vote in
    # the group baselines / normalisation ("include": every row votes)
    vm = sample_mask if cfg.get("masked_reward_policy", "include") == "exclude" else None
    adv = advantages_fn.compute_advantage(group_ids.view(-1, 1), rewards, token_mask,
                                          repeated_batch=rollout_batch, valid_mask=vm)
    if isinstance(adv, tuple):
        adv = adv[0]
    adv = adv.clone()
    lo, hi = cfg.get("advantage_clip_low"), cfg.get("advantage_clip_high")
    if lo is not None or hi is not None:
        adv = adv.clamp(min=lo, max=hi)
    gen_lp = flat.get("generation_logprobs", torch.zeros_like(token_mask)).float()
    data = BatchedDataDict({
        "input_ids": flat["token_ids"],
        "input_lengths": lengths,
        "advantages": adv * token_mask,
        "generation_logprobs": gen_lp,
        "token_mask": token_mask,
        "sample_mask": sample_mask,
    })
    data["rewards"] = rewards  # per-sample rewards (VAPO's positive-example NLL)
    apply_message_level_advantage_penalties(data, logs, cfg.get("invalid_tool_call_advantage"),
                                            cfg.get("malformed_thinking_advantage"))
    if cfg.get("invalid_tool_call_advantage") is not None or cfg.get("malformed_thinking_advantage") is not None:
        data["advantages"] = data["advantages"] * token_mask  # penalties only on trained tokens
    for k in ("sampler_topk_token_ids", "sampler_topk_logprobs"):  # score centering
        if k in flat:
            data[k] = flat[k]
    if "routed_experts" in flat:  # router replay (R3)
        data["routed_experts"] = flat["routed_experts"]
    stats = {"reward_mean": float(rewards.mean()), "reward_std": float(rewards.std()) if len(rewards) > 1 else 0.0,
             "advantage_abs_mean": float((adv.abs() * token_mask).sum() / token_mask.sum().clamp_min(1))}
    return data, stats


def _dp_sum(x: float, ps) -> float:
    if ps.dp_size <= 1:
        return x
    dev = ps.device if ps.device.type == "cuda" else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, group=ps.dp_group)
    return float(t.item())


def validate(policy, val_dataloader, val_task_to_env: dict, master_config: dict, step: int,
             tokenizer=None) -> dict:
    """Greedy (or val-temperature) rollouts over the validation set: mean reward
    ("accuracy") and pass@k over ``val_num_generations_per_prompt`` samples."""
    if val_dataloader is None:
        return {}
    cfg = {**DEFAULT_GRPO_CONFIG, **master_config.get("grpo", {})}
    k = int(cfg.get("val_num_generations_per_prompt", 1))
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    rewards_all, passk = [], []
    seen = 0
    policy.prepare_for_generation()
    for batch in val_dataloader:
        rep = batch.repeat_interleave(k)
        rollout, _ = run_multi_turn_rollout(policy, rep, tokenizer, val_task_to_env, max_seq,
                                            cfg.get("max_rollout_turns", 1), greedy=(k == 1))
        r = rollout["total_reward"]
        rewards_all.append(r)
        passk.append((r.view(-1, k) > 0).any(-1).float())
        seen += len(batch["message_log"])
        if seen >= cfg.get("max_val_samples", 256):
            break
    policy.finish_generation()
    if not rewards_all:
        return {}
    r = torch.cat(rewards_all)
    p = torch.cat(passk)
    return {"accuracy": float(r.mean()), "pass_k": float(p.mean()), "num_samples": int(r.numel())}


class _DeferredAdvantage:
    """Placeholder estimator for on-policy distillation: the advantages need the
    student's and the teachers' log-probs, so they are computed after those passes."""

    def compute_advantage(self, prompt_ids, rewards, mask, **_):
        return torch.zeros_like(mask, dtype=torch.float32)


def grpo_train(policy, dataloader, task_to_env: dict, master_config: dict, loss_fn=None, logger=None,
               checkpointer=None, save_state: Optional[GRPOSaveState] = None, val_dataloader=None,
               val_task_to_env: Optional[dict] = None, tokenizer=None, max_steps: Optional[int] = None,
               step_callback=None, teacher_router=None) -> GRPOSaveState:
    """Run GRPO steps; returns the final save state.  ``step_callback(step, metrics)``
    is called after every step (benchmarks hook timing there).  With
    ``on_policy_distillation.enabled`` (or ``adv_estimator.name: opd``) each step
    scores the rollouts with the routed teachers (``teacher_router``, built from
    the config when not given) and trains on the teacher-student log-prob gap."""
    ps = policy.ps
    cfg = {**DEFAULT_GRPO_CONFIG, **master_config.get("grpo", {})}
    loss_cfg = master_config.get("loss_fn", {})
    loss_fn = loss_fn or ClippedPGLossFn(loss_cfg)
    adv_cfg = dict(cfg.get("adv_estimator", {}) or {})
    adv_cfg.setdefault("normalize_rewards", cfg["normalize_rewards"])
    adv_cfg.setdefault("use_leave_one_out_baseline", cfg["use_leave_one_out_baseline"])
    estimator = make_advantage_estimator(adv_cfg, loss_cfg)
    from rl_b200.algorithms.opd import build_teacher_router, get_opd_full_config, is_opd_enabled, routing_keys

    opd = is_opd_enabled(master_config) or adv_cfg.get("name") == "opd"
    opd_full = get_opd_full_config(master_config) if opd else None
    if opd:
        if adv_cfg.get("name") != "opd":
            estimator = make_advantage_estimator({**adv_cfg, "name": "opd"}, loss_cfg)
        teacher_router = teacher_router or build_teacher_router(master_config, policy)
    if opd_full is not None:
        # full-vocabulary MOPD: exact reverse KL to the routed teacher's distribution
        from rl_b200.algorithms.loss.loss_functions import DistillationLossFn

        loss_fn = DistillationLossFn({"kl_type": "reverse"})
        full_k = int(opd_full.get("top_k") or policy.model_cfg.vocab_size)
    G = int(cfg["num_generations_per_prompt"])
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    train_gbs = int(master_config["policy"].get("train_global_batch_size", cfg["num_prompts_per_step"] * G))
    local_gbs = max(1, train_gbs // max(1, ps.dp_size))
    kl_on = float(loss_cfg.get("reference_policy_kl_penalty", 0.0) or 0.0) != 0.0
    from rl_b200.data_plane import create_data_plane

    if getattr(loss_fn, "score_centering", False) and hasattr(policy, "engine"):
        # the rollout records the sampler's top-k of every generated token
        policy.engine.record_sampler_topk = int(loss_cfg.get("score_centering_topk", 8))

    data_plane = create_data_plane(master_config.get("data_plane"))
    if cfg.get("length_penalty") is not None:  # reject a malformed block before the first rollout
        cfg["length_penalty"] = LengthPenaltyConfig(cfg["length_penalty"])
    state = save_state or GRPOSaveState.default()
    max_steps = max_steps if max_steps is not None else int(cfg["max_num_steps"])
    set_seed(int(cfg["seed"]) + ps.dp_rank)
    timer = Timer()
    from rl_b200.utils.telemetry import Telemetry

    tcfg = master_config.get("telemetry") or {}
    _telemetry = Telemetry(tcfg.get("path"), rank=ps.rank, otlp_endpoint=tcfg.get("otlp_endpoint"),
                           resource={"rl.algorithm": "grpo"})
    if checkpointer is not None:
        checkpointer.telemetry = _telemetry
    model_cfg = getattr(getattr(policy, "model", None), "cfg", None)
    flop_tracker = FLOPTracker(model_cfg) if model_cfg is not None else None
    step = int(state["current_step"])
    if cfg.get("val_at_start") and step == 0 and val_dataloader is not None:
        vm = validate(policy, val_dataloader, val_task_to_env or task_to_env, master_config, step, tokenizer)
        if logger:
            logger.log_metrics(vm, step, prefix="validation")
    done = False
    for epoch in range(int(state["current_epoch"]), int(cfg["max_num_epochs"])):
        for batch in dataloader:
            if step >= max_steps:
                done = True
                break
            timer.reset()
            maybe_gpu_profile_step(step)
            t_step = time.perf_counter()
            with timer.time("total_step_time"), _telemetry.span("step", **{"rl.step": step}) as step_span:
                # ---- rollouts (with DAPO dynamic sampling) ----
                kept_batches = []
                gen_batches = 0
                rollout_metrics: dict = {}
                with timer.time("generation"):
                    cur = batch
                    while True:
                        rep = cur.repeat_interleave(G)
                        n_prompts = len(cur["message_log"])
                        base = (step * 1000 + gen_batches) * 1_000_000 + ps.dp_rank * n_prompts
                        rep["group_id"] = torch.arange(base, base + n_prompts).repeat_interleave(G)
                        policy.prepare_for_generation(len(rep["message_log"]))
                        rollout, rollout_metrics = run_multi_turn_rollout(
                            policy, rep, tokenizer, task_to_env, max_seq, int(cfg["max_rollout_turns"]))
                        if cfg.get("length_penalty") is not None:
                            rollout_metrics.update(apply_length_penalty_to_rollout(
                                rollout, cfg["length_penalty"], G, tokenizer))
                        gen_batches += 1
                        if not cfg.get("use_dynamic_sampling", False):
                            kept_batches.append(rollout)
                            break
                        vote = rollout["loss_multiplier"] if cfg.get("masked_reward_policy",
                                                                      "include") == "exclude" else None
                        keep = dynamic_sampling(rollout["total_reward"], rollout["group_id"], vote)
                        rows = torch.nonzero(keep).flatten().tolist()
                        if rows:
                            kept_batches.append(rollout.select_indices(rows))
                        n_kept = sum(len(b["message_log"]) for b in kept_batches)
                        target = n_prompts * G
                        if n_kept >= target or gen_batches >= int(cfg["dynamic_sampling_max_gen_batches"]):
                            break
                        cur = batch
                    policy.finish_generation()
                rollout = BatchedDataDict.from_batches(kept_batches) if len(kept_batches) > 1 else kept_batches[0]
                if cfg.get("use_dynamic_sampling", False):
                    target = len(batch["message_log"]) * G
                    if len(rollout["message_log"]) > target:
                        rollout = rollout.slice(0, target)
                # ---- advantages ----
                with timer.time("data_processing"):
                    train_data, adv_stats = build_train_data(rollout, _DeferredAdvantage() if opd else estimator,
                                                             cfg, loss_cfg, rollout["group_id"])
                    if data_plane is not None:
                        # the trainer consumes the step's samples from the data plane (the
                        # reference's TransferQueue flow); producer and consumer may be
                        # different processes sharing the plane
                        key = f"step{step}/dp{ps.dp_rank}"
                        data_plane.put("train", key, train_data)
                        train_data = data_plane.get("train", key)
                        data_plane.delete("train", key)
                # ---- logprobs ----
                # one optimizer step per rollout batch: the weights before the step are
                # the ones the step's own forward runs with, so the separate "previous
                # policy" pass is folded into training (exactly the same values)
                one_step = train_data.size <= min(local_gbs, train_data.size)
                # OPD needs the student's log-probs before training (its advantages)
                reuse_prev = bool(cfg.get("reuse_train_logprobs_as_prev", True)) and one_step and not opd
                with timer.time("policy_and_reference_logprobs"):
                    policy.prepare_for_lp_inference()
                    if reuse_prev:
                        train_data["prev_logprobs"] = torch.zeros_like(train_data["generation_logprobs"])
                    else:
                        train_data["prev_logprobs"] = policy.get_logprobs(train_data)["logprobs"]
                    if kl_on and not cfg.get("skip_reference_policy_logprobs_calculation", False):
                        train_data["reference_policy_logprobs"] = \
                            policy.get_reference_policy_logprobs(train_data)["reference_logprobs"]
                    elif kl_on:  # skipped: the KL sees the current policy as its own reference
                        train_data["reference_policy_logprobs"] = train_data["generation_logprobs"].clone()
                    if opd:
                        tlp = teacher_router.teacher_logprobs(train_data, routing_keys(rollout))
                        train_data["teacher_logprobs"] = tlp
                        tm = train_data["token_mask"]
                        adv = estimator.compute_advantage(rollout["group_id"].view(-1, 1), train_data["rewards"], tm,
                                                          logprobs_policy=train_data["prev_logprobs"].float(),
                                                          logprobs_teacher=tlp)
                        train_data["advantages"] = adv * tm
                        adv_stats.update(estimator.last_metrics)
                        adv_stats.update(teacher_router.last_metrics)
                        if opd_full is not None:
                            v, ix = teacher_router.teacher_topk(train_data, routing_keys(rollout), full_k)
                            train_data["teacher_topk_logprobs"], train_data["teacher_topk_indices"] = v, ix
                # ---- train ----
                with timer.time("policy_training"):
                    policy.prepare_for_training()
                    n_rows = train_data.size
                    gbs = min(local_gbs, n_rows)
                    train_results = policy.train(train_data, loss_fn, gbs=gbs, prev_from_current=reuse_prev)
                if getattr(policy, "draft", None) is not None:
                    with timer.time("draft_training"):
                        train_results["draft_loss"] = policy.train_draft(train_data)
                # ---- refit ----
                with timer.time("weight_sync"):
                    refit_policy_generation(policy)
            step_time = time.perf_counter() - t_step
            # ---- metrics ----
            tok = float(train_data["input_lengths"].sum())
            gen_tok = float(train_data["token_mask"].sum())
            tok_all = _dp_sum(tok, ps) if ps.dp_size > 1 else tok
            gen_all = _dp_sum(gen_tok, ps) if ps.dp_size > 1 else gen_tok
            step_time_max = max_over_ranks(step_time)
            world = max(1, ps.world_size)
            metrics = dict(train_results)
            if flop_tracker is not None:
                # model FLOPs of this rank's sequences (TP peers share them), summed over DP
                flop_tracker.reset()
                fwd = _dp_sum(flop_tracker.track(train_data["input_lengths"].tolist()), ps)
                n_fwd_lp = 2 if kl_on else 1
                t_train = max_over_ranks(timer.get_elapsed("policy_training"))
                metrics["train_mfu"] = mfu(3 * fwd, t_train, world)
                metrics["step_mfu"] = mfu((3 + n_fwd_lp) * fwd, step_time_max, world)
                metrics["train_tflops_per_gpu"] = 3 * fwd / max(t_train, 1e-9) / world / 1e12
            metrics.update(adv_stats)
            metrics.update({k: v for k, v in rollout_metrics.items() if isinstance(v, (int, float))})
            metrics.update({
                "total_tokens": tok_all,
                "generated_tokens": gen_all,
                "tokens_per_sec": tok_all / step_time_max,
                "tokens_per_sec_per_gpu": tok_all / step_time_max / world,
                "step_time_s": step_time_max,
            })
            timing = {k: v for k, v in timer.get_timing_metrics().items()}
            metrics.update(_telemetry.goodput(timing, step_time_max))
            _telemetry.record_stage_spans(timing, parent=step_span)
            _telemetry.flush()
            step += 1
            state["current_step"] = step
            state["total_steps"] = int(state.get("total_steps", 0)) + 1
            state["consumed_samples"] = int(state.get("consumed_samples", 0)) + len(batch["message_log"]) * ps.dp_size
            state["total_valid_tokens"] = int(state.get("total_valid_tokens", 0)) + int(gen_all)
            if logger:
                logger.log_metrics(metrics, step, prefix="train")
                logger.log_metrics(timing, step, prefix="timing/train")
            if step_callback is not None:
                step_callback(step, {**metrics, **{"timing/" + k: v for k, v in timing.items()}})
            # ---- validation / checkpoint ----
            val_period = int(cfg.get("val_period") or 0)
            val_start = int(cfg.get("val_start_at", -1) or -1)
            if val_dataloader is not None and val_period > 0 and step % val_period == 0 and step >= val_start:
                vm = validate(policy, val_dataloader, val_task_to_env or task_to_env, master_config, step, tokenizer)
                state["val_reward"] = vm.get("accuracy")
                if logger:
                    logger.log_metrics(vm, step, prefix="validation")
                thr = cfg.get("stop_at_validation_threshold")
                key = cfg.get("stop_at_validation_metric")
                if key and thr is not None and vm.get(key, -math.inf) >= float(thr):
                    done = True
            out_of_time = checkpointer is not None and checkpointer.deadline_reached()
            if checkpointer is not None and (checkpointer.should_save(step) or out_of_time):
                checkpointer.save(policy, state, dataloader, metrics, step)
            if out_of_time:  # saved before the wall-clock deadline; stop here
                done = True
            if done:
                break
        if done or step >= max_steps:
            break
        state["current_epoch"] = epoch + 1
    if cfg.get("val_at_end") and val_dataloader is not None:
        vm = validate(policy, val_dataloader, val_task_to_env or task_to_env, master_config, step, tokenizer)
        if logger:
            logger.log_metrics(vm, step, prefix="validation")
    return state
