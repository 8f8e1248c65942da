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
    ``sequence_length_pad_multiple``; optional ``max_sequences_per_bin``,
    ``pair_grouping_key`` and ``microbatch_order`` (``"packer"`` | ``"largest_first"``)."""


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
        # sequence packing is requested: per global batch, [start, end) row ranges
        # and the padded length / packed token count of each micro-batch.
        self.micro_batch_indices: Optional[list[list[list[int]]]] = None
        self.micro_batch_lengths: Optional[list[list[int]]] = None
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
        out.elem_counts_per_gb = self.elem_counts_per_gb
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

    def reorder_data(self, reorded_indices: Sequence[int]) -> None:
        """Put row ``j`` at position ``reorded_indices[j]`` (undoes the row order
        that ``shard_by_batch_size`` returns with dynamic batching / packing)."""
        inv = [0] * len(reorded_indices)
        for j, dst in enumerate(reorded_indices):
            inv[int(dst)] = j
        idx = torch.as_tensor(inv, dtype=torch.long)
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
    ) -> Union[list["BatchedDataDict"], tuple[list["BatchedDataDict"], list[int]]]:
        """Split into ``shards`` data-parallel shards.

        The global batch is cut into chunks of ``batch_size`` rows (one
        optimizer step each; default: one chunk) and every chunk is split over
        the shards, so each shard holds its rows chunk by chunk.

        * Plain: chunk ``c`` gives shard ``s`` its rows
          ``[c*B + s*B/shards, c*B + (s+1)*B/shards)``; returns the shards.
        * ``dynamic_batching_args`` (``max_tokens_per_microbatch``,
          ``sequence_length_round``, ``input_key``, ``input_lengths_key``): rows
          of each chunk are sorted by length and dealt round-robin to the shards
          (every shard gets rows of similar length); the micro-batch plan is the
          same on every shard (a position's length is the max over shards, so
          every rank runs the same number of micro-batches of the same padded
          shape).  Returns ``(shards, sorted_indices)``.
        * ``sequence_packing_args`` (``max_tokens_per_microbatch``,
          ``input_lengths_key``, ``algorithm``, ``sequence_length_pad_multiple``,
          optional ``max_sequences_per_bin``, ``pair_grouping_key``,
          ``microbatch_order``): each chunk is bin-packed into a multiple of
          ``shards`` bins, dealt round-robin; ``microbatch_order="largest_first"``
          runs each shard's bins largest-first (the caching allocator then
          carves the smaller micro-batches out of the first one's blocks).
          ``pair_grouping_key`` keeps rows with the same key (a preference pair)
          in one bin.  Returns ``(shards, sorted_indices)``.

        With a plan, ``micro_batch_indices[c]`` lists ``[start, end)`` row ranges
        of chunk ``c`` (relative to the chunk's first row on the shard) and
        ``micro_batch_lengths[c]`` their padded length (dynamic) or packed token
        count (packing); ``elem_counts_per_gb[c]`` is the chunk's row count on the
        shard.  ``from_batches(shards).reorder_data(sorted_indices)`` restores
        the input order.

        Reference: ``nemo_rl/distributed/batched_data_dict.py:491``.
        """
        n = self.size
        if dynamic_batching_args is not None and sequence_packing_args is not None:
            raise ValueError("dynamic batching and sequence packing are mutually exclusive")
        if batch_size is None:
            batch_size = n
        if n % batch_size != 0:
            raise ValueError(f"Total batch size ({n}) is not a multiple of batch_size ({batch_size})")
        if not allow_uneven_shards and batch_size % shards != 0:
            raise ValueError(f"Batch size ({batch_size}) is not a multiple of shards ({shards})")
        num_chunks = n // batch_size
        if sequence_packing_args is not None:
            return self._shard_packed(shards, batch_size, num_chunks, sequence_packing_args)
        per_shard = math.ceil(batch_size / shards)
        order = list(range(n))
        if dynamic_batching_args is not None:
            lens = self._lengths(dynamic_batching_args.get("input_lengths_key", "input_lengths"))
            order = []
            for c in range(num_chunks):
                lo = c * batch_size
                by_len = sorted(range(lo, lo + batch_size), key=lambda i: lens[i])
                for s in range(shards):
                    order.extend(by_len[s::shards])
        shard_rows: list[list[int]] = [[] for _ in range(shards)]
        for c in range(num_chunks):
            for s in range(shards):
                lo = c * batch_size + s * per_shard
                hi = min(c * batch_size + batch_size, lo + per_shard)
                shard_rows[s].extend(order[lo:max(lo, hi)])
        out = [self.select_indices(rows) for rows in shard_rows]
        if dynamic_batching_args is None:
            return out
        self._plan_dynamic_shards(out, num_chunks, per_shard, dynamic_batching_args)
        return out, [r for rows in shard_rows for r in rows]

    def _lengths(self, key: str) -> list[int]:
        v = self.data[key]
        return v.tolist() if isinstance(v, torch.Tensor) else [int(x) for x in v]

    def _plan_dynamic_shards(self, out: list["BatchedDataDict"], num_chunks: int, per_shard: int, args: dict) -> None:
        budget = int(args["max_tokens_per_microbatch"])
        rnd = int(args.get("sequence_length_round", 1))
        key = args.get("input_lengths_key", "input_lengths")
        in_key = args.get("input_key")
        width = None
        if in_key is not None and isinstance(self.data.get(in_key), torch.Tensor) and self.data[in_key].dim() > 1:
            width = self.data[in_key].shape[1]
        shard_lens = [sh._lengths(key) for sh in out]
        mbi: list[list[list[int]]] = []
        mbl: list[list[int]] = []
        for c in range(num_chunks):
            idx: list[list[int]] = []
            lens: list[int] = []
            cur_max = 0
            for p in range(per_shard):
                L = max((sl[c * per_shard + p] for sl in shard_lens if c * per_shard + p < len(sl)), default=1)
                L = _round_up(max(1, L), rnd)
                if width is not None:
                    L = min(L, width)
                if L > budget:
                    raise ValueError(f"a row of padded length {L} does not fit max_tokens_per_microbatch={budget}")
                new_max = max(cur_max, L)
                if idx and (idx[-1][1] - idx[-1][0] + 1) * new_max <= budget:
                    idx[-1][1] += 1
                    lens[-1] = cur_max = new_max
                else:
                    idx.append([p, p + 1])
                    lens.append(L)
                    cur_max = L
            mbi.append(idx)
            mbl.append(lens)
        for sh in out:
            sh.micro_batch_indices = [[list(r) for r in chunk] for chunk in mbi]
            sh.micro_batch_lengths = [list(x) for x in mbl]
            sh.elem_counts_per_gb = [chunk[-1][1] if chunk else 0 for chunk in mbi]

    def _shard_packed(self, shards: int, batch_size: int, num_chunks: int, args: dict):
        order_mode = args.get("microbatch_order")
        if order_mode not in (None, "packer", "largest_first"):
            raise ValueError(f"sequence packing microbatch_order must be 'packer' or 'largest_first', got {order_mode!r}")
        pad = int(args.get("sequence_length_pad_multiple", 1))
        budget = int(args["max_tokens_per_microbatch"])
        packer = get_packer(args.get("algorithm", "modified_first_fit_decreasing"), bin_capacity=budget,
                            min_bin_count=shards, bin_count_multiple=shards,
                            max_sequences_per_bin=args.get("max_sequences_per_bin"))
        lens = self._lengths(args.get("input_lengths_key", "input_lengths"))
        group_key = args.get("pair_grouping_key")
        groups = None
        if group_key is not None:
            if group_key not in self.data:
                raise KeyError(f"sequence_packing pair_grouping_key={group_key!r} is not present in the batch")
            gv = self.data[group_key]
            groups = gv.tolist() if isinstance(gv, torch.Tensor) else list(gv)
        shard_rows: list[list[int]] = [[] for _ in range(shards)]
        shard_mbi: list[list] = [[] for _ in range(shards)]
        shard_mbl: list[list] = [[] for _ in range(shards)]
        shard_cnt: list[list[int]] = [[] for _ in range(shards)]
        for c in range(num_chunks):
            lo = c * batch_size
            padded = [_round_up(max(1, lens[lo + i]), pad) for i in range(batch_size)]
            if groups is None:
                bins = packer.pack(padded)
            else:
                members: dict = {}
                for i in range(batch_size):
                    members.setdefault(int(groups[lo + i]), []).append(i)
                gids = sorted(members)
                glens = [sum(padded[i] for i in members[g]) for g in gids]
                for g, L in zip(gids, glens):
                    if L > budget:
                        raise ValueError(f"sequence_packing pair group {g} requires {L} tokens but "
                                         f"max_tokens_per_microbatch={budget}")
                bins = [[i for gi in b for i in members[gids[gi]]] for b in packer.pack(glens)]
            for s in range(shards):
                mine = bins[s::shards]
                if order_mode == "largest_first":
                    mine = sorted(mine, key=lambda b: sum(padded[i] for i in b), reverse=True)
                idx, tok, start = [], [], 0
                for b in mine:
                    shard_rows[s].extend(lo + i for i in b)
                    idx.append([start, start + len(b)])
                    tok.append(sum(padded[i] for i in b))
                    start += len(b)
                shard_mbi[s].append(idx)
                shard_mbl[s].append(tok)
                shard_cnt[s].append(start)
        out = []
        for s in range(shards):
            sh = self.select_indices(shard_rows[s])
            sh.micro_batch_indices, sh.micro_batch_lengths, sh.elem_counts_per_gb = shard_mbi[s], shard_mbl[s], shard_cnt[s]
            out.append(sh)
        return out, [r for rows in shard_rows for r in rows]

    def get_batch(self, batch_idx: int, batch_size: Optional[int] = None) -> "BatchedDataDict":
        """Rows of global batch ``batch_idx`` (with its micro-batch plan when the
        shard carries one; ``batch_size`` is needed otherwise)."""
        if self.elem_counts_per_gb is not None:
            lo = sum(self.elem_counts_per_gb[:batch_idx])
            out = self.slice(lo, lo + self.elem_counts_per_gb[batch_idx])
            out.micro_batch_indices = [self.micro_batch_indices[batch_idx]]
            out.micro_batch_lengths = [self.micro_batch_lengths[batch_idx]]
            out.elem_counts_per_gb = [self.elem_counts_per_gb[batch_idx]]
            return out
        if batch_size is None:
            raise ValueError("get_batch needs batch_size when the batch has no micro-batch plan")
        return self.slice(batch_idx * batch_size, (batch_idx + 1) * batch_size)

    # -------------------------------------------------------------- iteration
    def make_microbatch_iterator(self, microbatch_size: int) -> Iterator["BatchedDataDict"]:
        n = self.size
        for start in range(0, n, microbatch_size):
            yield self.slice(start, min(n, start + microbatch_size))

    def _planned(self) -> Iterator[tuple[int, int, int]]:
        if self.micro_batch_indices is None:
            raise RuntimeError("no micro-batch plan; call shard_by_batch_size(dynamic_batching_args=... or "
                               "sequence_packing_args=...)")
        base = 0
        for c, (chunk, lens) in enumerate(zip(self.micro_batch_indices, self.micro_batch_lengths)):
            for (s, e), L in zip(chunk, lens):
                yield base + s, base + e, L
            base += self.elem_counts_per_gb[c] if self.elem_counts_per_gb is not None else (chunk[-1][1] if chunk else 0)

    def make_microbatch_iterator_with_dynamic_shapes(self, sequence_dim: int = 1) -> Iterator["BatchedDataDict"]:
        """Yield the planned micro-batches, each truncated to its padded length."""
        for s, e, L in self._planned():
            mb = self.slice(s, e)
            mb.truncate_tensors(sequence_dim, L)
            yield mb

    def get_microbatch_iterator_dynamic_shapes_len(self) -> int:
        return sum(len(c) for c in self.micro_batch_indices or [])

    def make_microbatch_iterator_for_packable_sequences(self) -> Iterator["BatchedDataDict"]:
        """Yield the planned packed micro-batches (rows to be concatenated THD-style)."""
        for s, e, _ in self._planned():
            yield self.slice(s, e)

    def get_microbatch_iterator_for_packable_sequences_len(self) -> tuple[int, int]:
        """(number of packed micro-batches, largest packed token count)."""
        lens = [L for c in self.micro_batch_lengths or [] for L in c]
        return len(lens), max(lens, default=0)

    def get_microbatch_iterator_len(self) -> int:
        return sum(len(c) for c in self.micro_batch_indices or [])

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
