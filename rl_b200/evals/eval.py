"""pass@k / cons@k evaluation with the in-house rollout engine.

Reference: ``eval_pass_k`` (``nemo_rl/evals/eval.py:178``), ``eval_cons_k``
(``:206``) and ``run_env_eval`` (``:280``).  Both scores are SUMS over prompts
(the caller divides by the prompt count), computed per group of
``num_tests_per_prompt`` consecutive samples:

* pass@k - the unbiased estimator 1 - C(n-c, k) / C(n, k) (n samples, c correct),
  evaluated as a product of (1 - k / j) for j = n-c+1 .. n;
* cons@k - the fraction of k-subsets of the n samples whose majority answer
  (ties: the answer seen first in the subset) is rewarded 1.0.  Subsets are
  enumerated exactly while C(n, k) <= ``max_subsets``; beyond that a fixed-seed
  sample of ``max_subsets`` subsets estimates the same fraction.
"""

from __future__ import annotations

import itertools
import math
import random
from collections import Counter
from typing import Optional, Sequence

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["eval_pass_k", "eval_cons_k", "run_env_eval"]


def _pass_at_k(n: int, c: int, k: int) -> float:
    if n - c < k:
        return 1.0
    prod = 1.0
    for j in range(n - c + 1, n + 1):
        prod *= 1.0 - k / j
    return 1.0 - prod


def eval_pass_k(rewards: torch.Tensor, num_tests_per_prompt: int, k: int) -> float:
    r = rewards.flatten().float()
    total = 0.0
    for g in r.split(num_tests_per_prompt):
        total += _pass_at_k(g.numel(), int((g == 1.0).sum()), k)
    return total


def _majority(answers: Sequence) -> object:
    cnt = Counter(answers)
    top = max(cnt.values())
    for a in answers:  # first answer reaching the top count
        if cnt[a] == top:
            return a
    return None


def eval_cons_k(rewards: torch.Tensor, num_tests_per_prompt: int, k: int, extracted_answers: Sequence,
                max_subsets: int = 20000, seed: int = 0) -> float:
    r = rewards.flatten().float().tolist()
    if len(extracted_answers) != len(r):
        raise ValueError("one extracted answer per reward expected")
    total = 0.0
    for g0 in range(0, len(r), num_tests_per_prompt):
        rw = r[g0:g0 + num_tests_per_prompt]
        ans = list(extracted_answers[g0:g0 + num_tests_per_prompt])
        n = len(ans)
        if n == 0 or k > n:
            continue
        if math.comb(n, k) <= max_subsets:
            subsets = itertools.combinations(range(n), k)
            count = math.comb(n, k)
        else:
            rng = random.Random(seed + g0)
            subsets = (sorted(rng.sample(range(n), k)) for _ in range(max_subsets))
            count = max_subsets
        ok = 0
        for sub in subsets:
            maj = _majority([ans[i] for i in sub])
            ok += rw[ans.index(maj)] == 1.0
        total += ok / count
    return total


def run_env_eval(policy, dataloader, env, master_config: dict, tokenizer=None,
                 answer_key: Optional[str] = "extracted_answer") -> dict:
    """Generate ``num_tests_per_prompt`` samples per prompt, score them with the
    environment and report ``eval.metric`` (``pass@k`` or ``cons@k``) averaged over
    prompts (``eval.k_value``; greedy when ``num_tests_per_prompt`` is 1)."""
    from rl_b200.experience.rollouts import run_multi_turn_rollout

    ecfg = master_config.get("eval", {})
    metric = ecfg.get("metric", "pass@k")
    if metric not in ("pass@k", "cons@k"):
        raise ValueError(f"unknown metric {metric}")
    n = int(ecfg.get("num_tests_per_prompt", 1))
    k = int(ecfg.get("k_value", 1))
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    task_to_env = env if isinstance(env, dict) else {"default": env}
    score, prompts, rewards_all = 0.0, 0, []
    policy.prepare_for_generation()
    for batch in dataloader:
        rep = batch.repeat_interleave(n) if isinstance(batch, BatchedDataDict) else batch
        rollout, _ = run_multi_turn_rollout(policy, rep, tokenizer, task_to_env, max_seq,
                                            int(ecfg.get("max_rollout_turns", 1)), greedy=(n == 1))
        r = rollout["total_reward"]
        rewards_all.append(r)
        prompts += len(batch["message_log"])
        if metric == "pass@k":
            score += eval_pass_k(r, n, k)
        else:
            infos = rollout.get("extra_env_info") or [None] * len(r)
            answers = [(i or {}).get(answer_key) if isinstance(i, dict) else None for i in infos]
            score += eval_cons_k(r, n, k, answers)
    policy.finish_generation()
    return {metric: score / max(1, prompts), "num_prompts": prompts,
            "mean_reward": float(torch.cat(rewards_all).mean()) if rewards_all else 0.0}
