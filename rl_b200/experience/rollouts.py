"""Rollout driver: generate -> environment step -> append, for one or more turns.

Reference: ``run_multi_turn_rollout`` (``nemo_rl/experience/rollouts.py:1031``),
``generate_responses`` (``:660``) and ``calculate_rewards`` (``:896``).  Each
turn flattens the active message logs, generates with the policy's rollout
engine, appends the assistant message (token ids + generation logprobs),
steps every task's environment, appends environment observations for samples
that continue, and accumulates rewards.
"""

from __future__ import annotations

import time
from typing import Any, Callable, Optional

import torch

from rl_b200.data.llm_message_utils import batched_message_log_to_flat_message
from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["generate_responses", "calculate_rewards", "run_multi_turn_rollout", "attach_routes"]


def generate_responses(policy_generation, batch: BatchedDataDict, rows: list[int], max_seq_len: int,
                       greedy: bool = False) -> tuple[list[torch.Tensor], list[torch.Tensor], list[bool], dict]:
    logs = [batch["message_log"][r] for r in rows]
    flat, lengths = batched_message_log_to_flat_message(logs)
    gen_in = BatchedDataDict({"input_ids": flat["token_ids"], "input_lengths": lengths})
    t0 = time.perf_counter()
    out = policy_generation.generate(gen_in, greedy=greedy)
    dt = time.perf_counter() - t0
    resp_ids, resp_lps, truncated = [], [], []
    for i in range(len(rows)):
        L = int(lengths[i])
        g = int(out["generation_lengths"][i])
        resp_ids.append(out["output_ids"][i, L:L + g].clone())
        resp_lps.append(out["logprobs"][i, L:L + g].clone())
        truncated.append(bool(out["truncated"][i]))
    stats = {"gen_time_s": dt, "gen_tokens": int(out["generation_lengths"].sum()),
             "prompt_tokens": int(lengths.sum())}
    if "sampler_topk_logprobs" in out:
        stats["sampler_topk"] = [(out["sampler_topk_token_ids"][i, int(lengths[i]):int(lengths[i]) +
                                                              int(out["generation_lengths"][i])],
                                  out["sampler_topk_logprobs"][i, int(lengths[i]):int(lengths[i]) +
                                                               int(out["generation_lengths"][i])])
                                 for i in range(len(rows))]
    if "routed_experts" in out:
        # router replay: the routes of every position of every generated sequence
        stats["routed_experts"] = [out["routed_experts"][i, :int(lengths[i]) + int(out["generation_lengths"][i])]
                                   for i in range(len(rows))]
    return resp_ids, resp_lps, truncated, stats


def attach_routes(log: list[dict], routes: torch.Tensor) -> None:
    """Give every message of ``log`` its slice of the full-sequence routes of
    the latest generation call (router replay; later turns overwrite earlier
    ones, so each token keeps the route of the last forward that processed it)."""
    off = 0
    for msg in log:
        L = len(msg["token_ids"])
        msg["routed_experts"] = routes[off:off + L].clone()
        off += L


def calculate_rewards(batch: BatchedDataDict, rows: list[int], task_to_env: dict) -> tuple[torch.Tensor, list, list]:
    """Group rows by task, step each task's environment once."""
    rewards = torch.zeros(len(rows), dtype=torch.float32)
    terminated = [True] * len(rows)
    observations: list[Any] = [None] * len(rows)
    by_task: dict[str, list[int]] = {}
    for i, r in enumerate(rows):
        by_task.setdefault(batch["task_name"][r], []).append(i)
    for task, idxs in by_task.items():
        env = task_to_env.get(task) or task_to_env.get("default")
        if env is None:
            raise KeyError(f"no environment registered for task {task!r}")
        logs = [batch["message_log"][rows[i]] for i in idxs]
        meta = [batch["extra_env_info"][rows[i]] for i in idxs]
        ret = env.step(logs, meta)
        for j, i in enumerate(idxs):
            rewards[i] = float(ret.rewards[j])
            terminated[i] = bool(ret.terminateds[j])
            observations[i] = ret.observations[j]
            batch["extra_env_info"][rows[i]] = ret.metadata[j]
    return rewards, terminated, observations


def run_multi_turn_rollout(policy_generation, input_batch: BatchedDataDict, tokenizer: Optional[Callable],
                           task_to_env: dict, max_seq_len: int, max_rollout_turns: int = 1, greedy: bool = False
                           ) -> tuple[BatchedDataDict, dict]:
    """Roll out every sample for up to ``max_rollout_turns`` turns.

    ``tokenizer`` (callable text -> token ids) is only needed for multi-turn
    environments whose observations carry text."""
    batch = input_batch.copy()
    B = len(batch["message_log"])
    batch["message_log"] = [[dict(m) for m in log] for log in batch["message_log"]]
    batch["extra_env_info"] = list(batch.get("extra_env_info", [None] * B))
    total_reward = torch.zeros(B, dtype=torch.float32)
    truncated = torch.zeros(B, dtype=torch.bool)
    active = list(range(B))
    metrics = {"gen_time_s": 0.0, "gen_tokens": 0, "turns": 0}
    for turn in range(max_rollout_turns):
        if not active:
            break
        # drop samples that already fill the context
        lens = {r: sum(len(m["token_ids"]) for m in batch["message_log"][r]) for r in active}
        live = [r for r in active if lens[r] < max_seq_len]
        for r in active:
            if r not in live:
                truncated[r] = True
        if not live:
            break
        resp, lps, trunc, st = generate_responses(policy_generation, batch, live, max_seq_len, greedy)
        metrics["gen_time_s"] += st["gen_time_s"]
        metrics["gen_tokens"] += st["gen_tokens"]
        metrics["turns"] += 1
        for i, r in enumerate(live):
            batch["message_log"][r].append({
                "role": "assistant", "content": "", "token_ids": resp[i],
                "generation_logprobs": lps[i],
            })
            if "routed_experts" in st:
                attach_routes(batch["message_log"][r], st["routed_experts"][i])
            if "sampler_topk" in st:
                msg = batch["message_log"][r][-1]
                msg["sampler_topk_token_ids"], msg["sampler_topk_logprobs"] = st["sampler_topk"][i]
            truncated[r] |= trunc[i]
        rewards, terminated, obs = calculate_rewards(batch, live, task_to_env)
        total_reward[torch.tensor(live)] += rewards
        nxt = []
        for i, r in enumerate(live):
            if terminated[i] or turn == max_rollout_turns - 1:
                continue
            o = obs[i] or {}
            text = o.get("content", "")
            if text and tokenizer is not None:
                ids = torch.tensor(tokenizer(text), dtype=torch.int64)
                batch["message_log"][r].append({"role": o.get("role", "environment"), "content": text,
                                                "token_ids": ids})
            nxt.append(r)
        active = nxt
    batch["total_reward"] = total_reward
    batch["truncated"] = truncated
    gen_lens = torch.tensor([sum(len(m["token_ids"]) for m in log if m["role"] == "assistant")
                             for log in batch["message_log"]], dtype=torch.float32)
    metrics.update({
        "mean_gen_tokens_per_sample": float(gen_lens.mean()) if B else 0.0,
        "max_gen_tokens": float(gen_lens.max()) if B else 0.0,
        "mean_total_reward": float(total_reward.mean()) if B else 0.0,
        "truncation_rate": float(truncated.float().mean()) if B else 0.0,
    })
    return batch, metrics
