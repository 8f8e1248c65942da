"""Deterministic synthetic reward environments for benchmarks and plumbing runs.

* ``EvenTokenEnvironment``: reward = fraction of generated token ids that are
  even (the tiny CPU GRPO configuration).
* ``HashRewardEnvironment``: reward in {0, 1} from a seeded polynomial rolling
  hash of the response token ids modulo the Mersenne prime 2^31 - 1 (the
  large-model benchmark configurations); deterministic across runs, ranks and
  hardware, and vectorised over the batch (one pass over token positions).
"""

from __future__ import annotations

from typing import Any

import torch

from rl_b200.environments.interfaces import EnvironmentInterface, EnvironmentReturn

__all__ = ["EvenTokenEnvironment", "HashRewardEnvironment", "hash_reward", "hash_rewards_batched", "response_tokens"]


def response_tokens(log: list[dict]) -> torch.Tensor:
    parts = [m["token_ids"] for m in log if m["role"] == "assistant"]
    return torch.cat(parts) if parts else torch.zeros(0, dtype=torch.int64)


_P = (1 << 31) - 1
_BASE = 1000003


def hash_rewards_batched(tokens: torch.Tensor, lengths: torch.Tensor, seed: int = 0) -> torch.Tensor:
    """``tokens [B, L]`` (right-padded), ``lengths [B]`` -> rewards ``[B]`` in {0, 1}."""
    B, L = tokens.shape
    h = torch.full((B,), (seed * 2654435761 + 12345) % _P, dtype=torch.int64)
    t = tokens.to(torch.int64) % _P
    for j in range(L):
        live = j < lengths
        nh = (h * _BASE + t[:, j] + 1) % _P
        h = torch.where(live, nh, h)
    return ((h >> 15) & 1).to(torch.float32)


def hash_reward(tokens: torch.Tensor, seed: int = 0) -> float:
    return float(hash_rewards_batched(tokens.view(1, -1), torch.tensor([tokens.numel()]), seed)[0])


class EvenTokenEnvironment(EnvironmentInterface):
    def __init__(self, cfg: dict | None = None):
        self.cfg = cfg or {}

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        rewards = []
        for log in message_log_batch:
            r = response_tokens(log)
            rewards.append(float((r % 2 == 0).float().mean()) if r.numel() else 0.0)
        n = len(message_log_batch)
        return EnvironmentReturn(
            observations=[{"role": "environment", "content": ""} for _ in range(n)],
            metadata=list(metadata), next_stop_strings=[None] * n,
            rewards=torch.tensor(rewards, dtype=torch.float32), terminateds=torch.ones(n, dtype=torch.bool),
            answers=[None] * n)


class HashRewardEnvironment(EnvironmentInterface):
    def __init__(self, cfg: dict | None = None):
        self.cfg = cfg or {}
        self.seed = int(self.cfg.get("seed", 0))

    def step(self, message_log_batch, metadata) -> EnvironmentReturn:
        resp = [response_tokens(log) for log in message_log_batch]
        n = len(message_log_batch)
        lens = torch.tensor([r.numel() for r in resp], dtype=torch.int64)
        padded = torch.zeros(n, int(lens.max()) if n else 0, dtype=torch.int64)
        for i, r in enumerate(resp):
            padded[i, : r.numel()] = r
        rewards = hash_rewards_batched(padded, lens, self.seed)
        return EnvironmentReturn(
            observations=[{"role": "environment", "content": ""} for _ in range(n)],
            metadata=list(metadata), next_stop_strings=[None] * n,
            rewards=rewards, terminateds=torch.ones(n, dtype=torch.bool),
            answers=[None] * n)
