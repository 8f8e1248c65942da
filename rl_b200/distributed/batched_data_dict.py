"""``BatchedDataDict``: the batch container passed between algorithm, policy and rollout code.

Behaviour follows the reference container (``nemo_rl/distributed/batched_data_dict.py:152``):
a ``dict`` whose tensor / list values share a leading batch dimension, with helpers
to shard a global batch over data-parallel ranks (``shard_by_batch_size`` ``:491``),
re-assemble it (``from_batches`` ``:243``) and iterate micro-batches, including
token-budgeted dynamic batching and sequence packing (``make_microbatch_iterator*``
``:1091-1150``).

Design notes (B200 build): batches here live on one rank at a time (the
framework is SPMD, one process per GPU), so the container is a thin layer over
tensors; micro-batch plans are computed once per global batch on the host and
stored as index lists so that the iterators never copy more than the rows they
emit.
"""

from __future__ import annotations

import math
from collections import UserDict
from typing import Any, Generic, Iterator, Optional, Sequence, TypeVar, Union

import torch

from rl_b200.data.packing import get_packer

T = TypeVar("T")

__all__ = ["BatchedDataDict", "DynamicBatchingArgs", "SequencePackingArgs"]


class DynamicBatchingArgs(dict):
    """Keys: ``max_tokens_per_microbatch``, ``sequence_length_round``, ``input_key``, ``input_lengths_key``."""


class SequencePackingArgs(dict):
    """Keys: ``max_tokens_per_microbatch``, ``input_key``, ``input_lengths_key``, ``algorithm``,
    ``sequence_length_pad_multiple``."""


def _batch_len(v: Any) -> int:
    if isinstance(v, torch.Tensor):
        return 0 if v.dim() == 0 else v.shape[0]
    return len(v)


def _index(v: Any, idx: Union[torch.Tensor, Sequence[int], slice]) -> Any:
    if isinstance(v, torch.Tensor):
        if isinstance(idx, slice):
            return v[idx]
        if not isinstance(idx, torch.Tensor):
            idx = torch.as_tensor(list(idx), dtype=torch.long)
        return v.index_select(0, idx.to(v.device))
    if isinstance(idx, slice):
        return v[idx]
    if isinstance(idx, torch.Tensor):
        idx = idx.tolist()
    return [v[i] for i in idx]


class BatchedDataDict(UserDict, Generic[T]):
    """Dictionary of batch-major tensors and lists."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        # Micro-batch plan produced by shard_by_batch_size when dynamic batching or
        # sequence packing is requested: list of index lists, one per micro-batch,
        # plus the padded sequence length of each micro-batch.
        self.micro_batch_indices: Optional[list[list[int]]] = None
        self.micro_batch_lengths: Optional[list[int]] = None
        self.elem_counts_per_gb: Optional[list[int]] = None

    # ------------------------------------------------------------------ basics
    @property
    def size(self) -> int:
        sizes = {_batch_len(v) for v in self.data.values() if isinstance(v, (torch.Tensor, list, tuple))}
        sizes.discard(0)
        if not sizes:
            return 0
        if len(sizes) != 1:
            raise ValueError(f"inconsistent batch sizes in BatchedDataDict: { {k: _batch_len(v) for k, v in self.data.items()} }")
        return sizes.pop()

    def get_dict(self) -> dict:
        return dict(self.data)

    def copy(self) -> "BatchedDataDict":
        out = type(self)(dict(self.data))
        out.micro_batch_indices = self.micro_batch_indices
        out.micro_batch_lengths = self.micro_batch_lengths
        return out

    def to(self, device: Union[str, torch.device], non_blocking: bool = False) -> "BatchedDataDict":
        for k, v in self.data.items():
            if isinstance(v, torch.Tensor):
                self.data[k] = v.to(device, non_blocking=non_blocking)
        return self

    def pin_memory(self) -> "BatchedDataDict":
        for k, v in self.data.items():
            if isinstance(v, torch.Tensor) and v.device.type == "cpu":
                self.data[k] = v.pin_memory()
        return self

    def select_indices(self, indices: Union[torch.Tensor, Sequence[int]]) -> "BatchedDataDict":
        return type(self)({k: _index(v, indices) for k, v in self.data.items()})

    def slice(self, start: int, end: int) -> "BatchedDataDict":
        return type(self)({k: _index(v, slice(start, end)) for k, v in self.data.items()})

    def get_batch(self, batch_idx: int, batch_size: int) -> "BatchedDataDict":
        return self.slice(batch_idx * batch_size, (batch_idx + 1) * batch_size)

    def reorder_data(self, order: Sequence[int]) -> None:
        idx = torch.as_tensor(list(order), dtype=torch.long)
        for k, v in list(self.data.items()):
            self.data[k] = _index(v, idx)

    def repeat_interleave(self, num_repeats: int) -> "BatchedDataDict":
        out = {}
        for k, v in self.data.items():
            if isinstance(v, torch.Tensor):
                out[k] = v.repeat_interleave(num_repeats, dim=0)
            else:
                out[k] = [x for x in v for _ in range(num_repeats)]
        return type(self)(out)

    def truncate_tensors(self, dim: int, truncated_len: int) -> None:
        for k, v in self.data.items():
            if isinstance(v, torch.Tensor) and v.dim() > dim:
                self.data[k] = v.narrow(dim, 0, min(truncated_len, v.shape[dim]))

    def chunk(self, rank: int, chunks: int) -> "BatchedDataDict":
        n = self.size
        per = math.ceil(n / chunks)
        return self.slice(rank * per, min(n, (rank + 1) * per))

    # ------------------------------------------------------------- assembling
    @classmethod
    def from_batches(
        cls, batches: Sequence["BatchedDataDict"], pad_value_dict: Optional[dict[str, Any]] = None
    ) -> "BatchedDataDict":
        """Concatenate batches along dim 0; 2-D+ tensors are right-padded to the widest.

        ``pad_value_dict`` maps a key to its pad value (default 0).
        """
        pad_value_dict = pad_value_dict or {}
        if not batches:
            return cls()
        keys = list(batches[0].keys())
        out = {}
        for k in keys:
            vals = [b[k] for b in batches]
            if isinstance(vals[0], torch.Tensor):
                if vals[0].dim() >= 2:
                    width = max(v.shape[1] for v in vals)
                    padded = []
                    for v in vals:
                        if v.shape[1] < width:
                            pad_shape = list(v.shape)
                            pad_shape[1] = width - v.shape[1]
                            pad = torch.full(pad_shape, pad_value_dict.get(k, 0), dtype=v.dtype, device=v.device)
                            v = torch.cat([v, pad], dim=1)
                        padded.append(v)
                    vals = padded
                out[k] = torch.cat(vals, dim=0) if vals[0].dim() > 0 else torch.stack(vals)
            else:
                merged: list = []
                for v in vals:
                    merged.extend(v)
                out[k] = merged
        return cls(out)

    def all_gather(self, group=None) -> "BatchedDataDict":
        """Gather every rank's batch (object collective; used for small host-side data)."""
        import torch.distributed as dist

        world = dist.get_world_size(group)
        gathered: list = [None] * world
        cpu = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in self.data.items()}
        dist.all_gather_object(gathered, cpu, group=group)
        return type(self).from_batches([type(self)(g) for g in gathered])

    # ---------------------------------------------------------------- sharding
    def shard_by_batch_size(
        self,
        shards: int,
        batch_size: Optional[int] = None,
        allow_uneven_shards: bool = False,
        dynamic_batching_args: Optional[dict] = None,
        sequence_packing_args: Optional[dict] = None,
    ) -> list["BatchedDataDict"]:
        """Split into ``shards`` data-parallel shards.

        With ``batch_size`` set, the global batch is first cut into chunks of
        ``batch_size`` rows (one optimizer step each) and every chunk is split
        evenly over the shards, so each shard holds ``size/shards`` rows ordered
        chunk by chunk - the layout the reference's ``shard_by_batch_size``
        produces.  With dynamic batching or sequence packing the rows of each
        chunk are also planned into token-budgeted micro-batches (stored on each
        shard as ``micro_batch_indices``).
        """
        n = self.size
        if dynamic_batching_args is not None and sequence_packing_args is not None:
            raise ValueError("dynamic batching and sequence packing are mutually exclusive")
        if batch_size is None:
            batch_size = n
        if n % batch_size != 0:
            raise ValueError(f"batch size {n} is not a multiple of batch_size {batch_size}")
        if not allow_uneven_shards and batch_size % shards != 0:
            raise ValueError(f"batch_size {batch_size} is not divisible by {shards} shards")
        per_shard = math.ceil(batch_size / shards)
        shard_rows: list[list[int]] = [[] for _ in range(shards)]
        for chunk_start in range(0, n, batch_size):
            for s in range(shards):
                lo = chunk_start + s * per_shard
                hi = min(chunk_start + batch_size, lo + per_shard)
                shard_rows[s].extend(range(lo, max(lo, hi)))
        out = [self.select_indices(rows) for rows in shard_rows]
        rows_per_gb = per_shard
        if dynamic_batching_args is not None or sequence_packing_args is not None:
            args = dynamic_batching_args or sequence_packing_args
            lengths_key = args.get("input_lengths_key", "input_lengths")
            for shard in out:
                lengths = shard[lengths_key]
                lengths = lengths.tolist() if isinstance(lengths, torch.Tensor) else list(lengths)
                mbs: list[list[int]] = []
                mb_lens: list[int] = []
                counts: list[int] = []
                for gb_start in range(0, len(lengths), rows_per_gb):
                    gb_rows = list(range(gb_start, min(len(lengths), gb_start + rows_per_gb)))
                    gb_lens = [lengths[i] for i in gb_rows]
                    if sequence_packing_args is not None:
                        plan = _plan_packing(gb_rows, gb_lens, sequence_packing_args)
                    else:
                        plan = _plan_dynamic(gb_rows, gb_lens, dynamic_batching_args)
                    for rows, L in plan:
                        mbs.append(rows)
                        mb_lens.append(L)
                    counts.append(len(plan))
                shard.micro_batch_indices = mbs
                shard.micro_batch_lengths = mb_lens
                shard.elem_counts_per_gb = counts
        return out

    # -------------------------------------------------------------- iteration
    def make_microbatch_iterator(self, microbatch_size: int) -> Iterator["BatchedDataDict"]:
        n = self.size
        for start in range(0, n, microbatch_size):
            yield self.slice(start, min(n, start + microbatch_size))

    def make_microbatch_iterator_with_dynamic_shapes(self, sequence_dim: int = 1) -> Iterator["BatchedDataDict"]:
        """Yield the planned micro-batches, each truncated to its rounded max length."""
        if self.micro_batch_indices is None:
            raise RuntimeError("no dynamic micro-batch plan; call shard_by_batch_size(dynamic_batching_args=...)")
        for rows, L in zip(self.micro_batch_indices, self.micro_batch_lengths):
            mb = self.select_indices(rows)
            mb.truncate_tensors(sequence_dim, L)
            yield mb

    def make_microbatch_iterator_for_packable_sequences(self) -> Iterator["BatchedDataDict"]:
        """Yield the planned packed micro-batches (rows to be concatenated THD-style)."""
        if self.micro_batch_indices is None:
            raise RuntimeError("no packing plan; call shard_by_batch_size(sequence_packing_args=...)")
        for rows in self.micro_batch_indices:
            yield self.select_indices(rows)

    def get_microbatch_iterator_len(self) -> int:
        return 0 if self.micro_batch_indices is None else len(self.micro_batch_indices)

    def __repr__(self) -> str:  # pragma: no cover - debugging helper
        parts = []
        for k, v in self.data.items():
            if isinstance(v, torch.Tensor):
                parts.append(f"{k}: Tensor{tuple(v.shape)} {v.dtype}")
            else:
                parts.append(f"{k}: list[{len(v)}]")
        return "BatchedDataDict(" + ", ".join(parts) + ")"


def _round_up(x: int, m: int) -> int:
    return ((x + m - 1) // m) * m if m > 1 else x


def _plan_dynamic(rows: list[int], lengths: list[int], args: dict) -> list[tuple[list[int], int]]:
    """Greedy token-budget micro-batching: rows sorted by length, a batch closes when
    ``rows * round_up(max_len)`` would exceed the budget (reference semantics of
    ``dynamic_batching``: ``train_mb_tokens`` and ``sequence_length_round``)."""
    budget = int(args["max_tokens_per_microbatch"])
    rnd = int(args.get("sequence_length_round", 1))
    order = sorted(range(len(rows)), key=lambda i: lengths[i])
    plan: list[tuple[list[int], int]] = []
    cur: list[int] = []
    cur_max = 0
    for i in order:
        L = _round_up(max(1, lengths[i]), rnd)
        new_max = max(cur_max, L)
        if cur and new_max * (len(cur) + 1) > budget:
            plan.append(([rows[j] for j in cur], cur_max))
            cur, cur_max = [], 0
            new_max = L
        cur.append(i)
        cur_max = new_max
    if cur:
        plan.append(([rows[j] for j in cur], cur_max))
    return plan


def _plan_packing(rows: list[int], lengths: list[int], args: dict) -> list[tuple[list[int], int]]:
    budget = int(args["max_tokens_per_microbatch"])
    pad_mult = int(args.get("sequence_length_pad_multiple", 1))
    algorithm = args.get("algorithm", "modified_first_fit_decreasing")
    padded = [_round_up(max(1, L), pad_mult) for L in lengths]
    packer = get_packer(algorithm, bin_capacity=budget)
    bins = packer.pack(padded)
    plan = []
    for b in bins:
        plan.append(([rows[i] for i in b], sum(padded[i] for i in b)))
    return plan
