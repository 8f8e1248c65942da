"""Prompt datasets and a stateful data loader.

* ``SyntheticPromptDataset`` - prompts of uniform-random token ids with lengths
  uniform in ``[min_len, max_len]`` (the synthetic data of the benchmark
  configs: no network, no tokenizer).
* ``JsonlPromptDataset`` - ``{"problem"/"prompt", "answer"/"expected_answer"}``
  rows tokenised with a user-supplied tokenizer (math-style tasks).
* ``PreferenceDataset`` / ``SFTDataset`` - for DPO/RM and SFT loops.
* ``StatefulDataLoader`` - deterministic per-epoch shuffling with a
  ``state_dict`` for checkpoint/resume (reference: torchdata ``StatefulDataLoader``
  used at ``nemo_rl/algorithms/grpo.py:884``, dataloader state saved
  ``nemo_rl/data/utils.py:69,85``), sharded by data-parallel rank.
"""

from __future__ import annotations

import json
import random
from typing import Any, Callable, Iterator, Optional

import torch

from rl_b200.data.interfaces import DatumSpec

__all__ = ["SyntheticPromptDataset", "JsonlPromptDataset", "SFTDataset", "PreferenceDataset", "StatefulDataLoader",
           "rl_collate_fn"]


class SyntheticPromptDataset:
    def __init__(self, num_samples: int, min_len: int, max_len: int, vocab_size: int, seed: int = 0,
                 task_name: str = "synthetic", vocab_low: int = 0):
        self.n = num_samples
        self.min_len, self.max_len = min_len, max_len
        self.vocab = vocab_size
        self.vocab_low = vocab_low
        self.seed = seed
        self.task_name = task_name

    def __len__(self) -> int:
        return self.n

    def __getitem__(self, i: int) -> DatumSpec:
        g = torch.Generator().manual_seed(self.seed * 1000003 + i)
        L = int(torch.randint(self.min_len, self.max_len + 1, (1,), generator=g))
        ids = torch.randint(self.vocab_low, self.vocab, (L,), generator=g)
        return {
            "message_log": [{"role": "user", "content": "", "token_ids": ids}],
            "length": L,
            "extra_env_info": {"prompt_index": i},
            "loss_multiplier": 1.0,
            "idx": i,
            "task_name": self.task_name,
        }


class JsonlPromptDataset:
    def __init__(self, path: str, tokenize: Callable[[str], list[int]], prompt_template: str = "{}",
                 task_name: str = "math", max_len: Optional[int] = None):
        self.rows = [json.loads(l) for l in open(path) if l.strip()]
        self.tokenize = tokenize
        self.template = prompt_template
        self.task_name = task_name
        self.max_len = max_len

    def __len__(self):
        return len(self.rows)

    def __getitem__(self, i: int) -> DatumSpec:
        r = self.rows[i]
        text = self.template.format(r.get("problem", r.get("prompt", "")))
        ids = torch.tensor(self.tokenize(text), dtype=torch.int64)
        if self.max_len:
            ids = ids[: self.max_len]
        return {
            "message_log": [{"role": "user", "content": text, "token_ids": ids}],
            "length": int(ids.shape[0]),
            "extra_env_info": {"ground_truth": r.get("answer", r.get("expected_answer"))},
            "loss_multiplier": 1.0,
            "idx": i,
            "task_name": self.task_name,
        }


class SFTDataset:
    """Synthetic prompt/response pairs (or supplied token lists) for SFT."""

    def __init__(self, samples: list[tuple[list[int], list[int]]]):
        self.samples = samples

    def __len__(self):
        return len(self.samples)

    def __getitem__(self, i):
        p, r = self.samples[i]
        return {
            "message_log": [{"role": "user", "content": "", "token_ids": torch.tensor(p)},
                            {"role": "assistant", "content": "", "token_ids": torch.tensor(r)}],
            "length": len(p) + len(r), "loss_multiplier": 1.0, "idx": i, "task_name": "sft",
        }


class PreferenceDataset:
    """(prompt, chosen, rejected) token triples for DPO / reward modelling."""

    def __init__(self, samples: list[tuple[list[int], list[int], list[int]]]):
        self.samples = samples

    def __len__(self):
        return len(self.samples)

    def __getitem__(self, i):
        p, c, r = self.samples[i]
        return {"prompt": torch.tensor(p), "chosen": torch.tensor(c), "rejected": torch.tensor(r), "idx": i}


def rl_collate_fn(batch: list[DatumSpec]) -> dict:
    """Collate datum dicts into a batch of lists (message logs stay ragged)."""
    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    out = BatchedDataDict({
        "message_log": [b["message_log"] for b in batch],
        "length": torch.tensor([b["length"] for b in batch], dtype=torch.int64),
        "loss_multiplier": torch.tensor([b.get("loss_multiplier", 1.0) for b in batch], dtype=torch.float32),
        "extra_env_info": [b.get("extra_env_info") for b in batch],
        "task_name": [b.get("task_name", "default") for b in batch],
        "idx": torch.tensor([b.get("idx", i) for i, b in enumerate(batch)], dtype=torch.int64),
        "stop_strings": [b.get("stop_strings") for b in batch],
    })
    if any("packed_segments" in b for b in batch):  # packed Megatron SFT rows
        out["packed_segments"] = [b.get("packed_segments") for b in batch]
    return out


class StatefulDataLoader:
    """Deterministic, resumable batch iterator over an indexable dataset.

    ``shard_rank``/``num_shards`` split every global batch across data-parallel
    ranks (each rank sees ``batch_size // num_shards`` rows of the same global
    batch order)."""

    def __init__(self, dataset, batch_size: int, shuffle: bool = True, seed: int = 0, drop_last: bool = True,
                 collate_fn: Callable = rl_collate_fn, shard_rank: int = 0, num_shards: int = 1):
        if batch_size % num_shards:
            raise ValueError(f"batch size {batch_size} not divisible by {num_shards} data-parallel shards")
        self.dataset = dataset
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.seed = seed
        self.drop_last = drop_last
        self.collate_fn = collate_fn
        self.shard_rank, self.num_shards = shard_rank, num_shards
        self.epoch = 0
        self.batch_in_epoch = 0

    def _order(self) -> list[int]:
        idx = list(range(len(self.dataset)))
        if self.shuffle:
            random.Random(self.seed + self.epoch).shuffle(idx)
        return idx

    def __len__(self) -> int:
        n = len(self.dataset) // self.batch_size
        return n if self.drop_last else -(-len(self.dataset) // self.batch_size)

    def __iter__(self) -> Iterator[Any]:
        while True:
            order = self._order()
            nb = len(self)
            while self.batch_in_epoch < nb:
                b = self.batch_in_epoch
                rows = order[b * self.batch_size:(b + 1) * self.batch_size]
                per = len(rows) // self.num_shards
                mine = rows[self.shard_rank * per:(self.shard_rank + 1) * per]
                self.batch_in_epoch += 1
                yield self.collate_fn([self.dataset[i] for i in mine])
            self.epoch += 1
            self.batch_in_epoch = 0
            return

    def state_dict(self) -> dict:
        return {"epoch": self.epoch, "batch_in_epoch": self.batch_in_epoch, "seed": self.seed}

    def load_state_dict(self, sd: dict) -> None:
        self.epoch = int(sd["epoch"])
        self.batch_in_epoch = int(sd["batch_in_epoch"])
        self.seed = int(sd.get("seed", self.seed))
