"""Non-colocated GRPO: training and generation on different GPUs / processes.

Reference: ``policy.generation.colocated.enabled: false`` (``examples/configs/
grpo_math_1B.yaml:395-399``): the generation engine runs on its own resources,
and after every optimizer step the trainer broadcasts its weights to it
(``packed_broadcast_producer`` / consumer, ``nemo_rl/utils/packed_tensor.py``)
over a communicator that spans both sides.

Here the two sides are separate jobs (or separate rank sets of one job) that
share only:

* a key-value data plane (``StoreDataPlane`` on a TCPStore): the trainer puts
  each step's prompt batch under ``prompts/<step>``, the generator puts the
  rollout batch under ``rollouts/<step>``, and ``prompts/stop`` ends the
  generator;
* a two-member ``StatelessProcessGroup`` (trainer rank 0 = broadcast source,
  generator = consumer) over which ``PackedBroadcastSynchronizer`` streams the
  flat weight buffer in buckets straight into the generator's buffer.

Both sides build the same model configuration (same flat layout), so a refit is
the broadcast of one contiguous buffer.  With ``lead: 0`` (default) the step is
on-policy: the generator waits for the refit that follows step ``s`` before it
generates step ``s + 1``.  With ``lead: 1`` it generates step ``s + 1`` with the
weights of step ``s - 1`` while the trainer trains step ``s`` (one step stale, as
in async GRPO with ``max_trajectory_age_steps: 1``), and takes the refit after.
"""

from __future__ import annotations

import time
from typing import Optional

import torch

__all__ = ["noncolocated_grpo_train", "serve_generation"]

PROMPTS, ROLLOUTS = "prompts", "rollouts"


def _repeat(batch, G: int, step: int, rank: int):
    rep = batch.repeat_interleave(G)
    n = len(batch["message_log"])
    base = step * 1_000_000 + rank * 10_000
    rep["group_id"] = torch.arange(base, base + n).repeat_interleave(G)
    return rep


def noncolocated_grpo_train(policy, dataloader, master_config: dict, plane, sync, loss_fn=None, logger=None,
                            max_steps: Optional[int] = None, timeout_s: float = 3600.0) -> list[dict]:
    """Trainer side: ``policy`` a ``PolicyWorker`` that trains; ``plane`` a data
    plane shared with the generator; ``sync`` a ``PackedBroadcastSynchronizer``
    whose source is this process.  Returns the per-step metrics."""
    from rl_b200.algorithms.advantage_estimator import make_advantage_estimator
    from rl_b200.algorithms.grpo import DEFAULT_GRPO_CONFIG, build_train_data
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn

    cfg = {**DEFAULT_GRPO_CONFIG, **master_config.get("grpo", {})}
    loss_cfg = master_config.get("loss_fn", {})
    loss_fn = loss_fn or ClippedPGLossFn(loss_cfg)
    adv_cfg = dict(cfg.get("adv_estimator", {}) or {})
    adv_cfg.setdefault("normalize_rewards", cfg["normalize_rewards"])
    adv_cfg.setdefault("use_leave_one_out_baseline", cfg["use_leave_one_out_baseline"])
    estimator = make_advantage_estimator(adv_cfg, loss_cfg)
    G = int(cfg["num_generations_per_prompt"])
    kl_on = float(loss_cfg.get("reference_policy_kl_penalty", 0.0) or 0.0) != 0.0
    lead = int(((master_config["policy"].get("generation") or {}).get("colocated") or {}).get("lead", 0))
    steps = max_steps if max_steps is not None else int(cfg["max_num_steps"])
    it = iter(dataloader)
    history = []
    sync.sync()  # the generator starts from the trainer's initial weights
    for s in range(min(lead + 1, steps)):  # prompts the generator may work ahead on
        plane.put(PROMPTS, str(s), _repeat(next(it), G, s, 0))
    for step in range(steps):
        t0 = time.perf_counter()
        rollout = plane.get(ROLLOUTS, str(step), timeout=timeout_s)
        plane.delete(ROLLOUTS, str(step))
        nxt = step + lead + 1
        if nxt < steps:
            plane.put(PROMPTS, str(nxt), _repeat(next(it), G, nxt, 0))
        if step == steps - 1:
            # every prompt is out: the generator may finish, taking the refits still to come
            plane.put(PROMPTS, "stop", {"stop": torch.ones(1)})
        train_data, adv_stats = build_train_data(rollout, estimator, cfg, loss_cfg, rollout["group_id"])
        train_data["prev_logprobs"] = policy.get_logprobs(train_data)["logprobs"]
        if kl_on:
            train_data["reference_policy_logprobs"] = \
                policy.get_reference_policy_logprobs(train_data)["reference_logprobs"]
        res = policy.train(train_data, loss_fn)
        t_sync = time.perf_counter()
        stats = sync.sync()  # trainer -> generator weights (bucketed broadcast)
        m = {"loss": float(res["loss"]), "grad_norm": float(res["grad_norm"]),
             "reward_mean": float(rollout["total_reward"].float().mean()), **adv_stats,
             "timing/weight_sync": time.perf_counter() - t_sync, "step_time_s": time.perf_counter() - t0,
             "refit_bytes": float(stats["bytes"])}
        history.append(m)
        if logger:
            logger.log_metrics(m, step + 1, prefix="train")
    return history


def serve_generation(policy, master_config: dict, plane, sync, task_to_env: dict, tokenizer=None,
                     timeout_s: float = 3600.0) -> int:
    """Generator side: ``policy`` a ``PolicyWorker`` used for generation only;
    ``sync`` a ``PackedBroadcastSynchronizer`` consuming into its flat buffer.
    Serves steps until the trainer's stop marker; returns the steps served."""
    from rl_b200.algorithms.grpo import DEFAULT_GRPO_CONFIG
    from rl_b200.experience.rollouts import run_multi_turn_rollout

    cfg = {**DEFAULT_GRPO_CONFIG, **master_config.get("grpo", {})}
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    lead = int(((master_config["policy"].get("generation") or {}).get("colocated") or {}).get("lead", 0))

    refits = 0

    def refit():
        nonlocal refits
        sync.sync()
        policy.engine.update_weights_from_training()
        policy.engine.invalidate_kv_cache()
        refits += 1

    refit()  # initial weights
    step = 0
    while True:
        key = str(step)
        deadline = time.monotonic() + timeout_s
        while key not in plane.keys(PROMPTS) and "stop" not in plane.keys(PROMPTS):
            if time.monotonic() > deadline:
                raise TimeoutError(f"no prompts for step {step} within {timeout_s:.0f} s")
            time.sleep(0.002)
        if key not in plane.keys(PROMPTS):
            # stop marker: take the trainer's remaining refits (one per trained step
            # plus the initial one) so its last broadcasts complete
            while refits < step + 1:
                refit()
            return step
        batch = plane.get(PROMPTS, key, timeout=timeout_s)
        plane.delete(PROMPTS, key)
        policy.prepare_for_generation(len(batch["message_log"]))
        rollout, _ = run_multi_turn_rollout(policy, batch, tokenizer, task_to_env, max_seq,
                                            int(cfg["max_rollout_turns"]))
        plane.put(ROLLOUTS, key, rollout)
        if step >= lead:
            refit()  # the weights trained on step (step - lead)
        step += 1
