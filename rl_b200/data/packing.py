"""Bin-packing of variable-length sequences into token-budgeted micro-batches.

Offers the packers the reference exposes (``nemo_rl/data/packing/algorithms.py``:
concatenative ``:384``, first-fit ``:446``, first-fit-decreasing ``:516``,
first-fit-shuffle ``:544``, modified first-fit-decreasing ``:572``, greedy
knapsack ``:298``, balanced greedy knapsack ``:328``; factory ``get_packer``
``:759``).  Each packer maps a list of sequence lengths to bins (lists of indices)
whose summed length does not exceed ``bin_capacity``.

The modified first-fit-decreasing heuristic is the published one of Johnson &
Garey, "A 71/60 theorem for bin packing" (J. Complexity 1985): items are
classed large (>C/2), medium (>C/3), small (>C/6) and tiny; every large item
opens a bin, medium items are placed into large bins (largest-first), pairs of
small items fill the remaining gaps of bins without a medium item (scanning
from the fullest), and everything left is placed first-fit-decreasing.
"""

from __future__ import annotations

import enum
import random
from typing import Optional

__all__ = [
    "PackingAlgorithm",
    "SequencePacker",
    "ConcatenativePacker",
    "FirstFitPacker",
    "FirstFitDecreasingPacker",
    "FirstFitShufflePacker",
    "ModifiedFirstFitDecreasingPacker",
    "GreedyKnapsackPacker",
    "BalancedGreedyKnapsackPacker",
    "get_packer",
]


class PackingAlgorithm(enum.Enum):
    CONCATENATIVE = "concatenative"
    FIRST_FIT = "first_fit"
    FIRST_FIT_DECREASING = "first_fit_decreasing"
    FIRST_FIT_SHUFFLE = "first_fit_shuffle"
    MODIFIED_FIRST_FIT_DECREASING = "modified_first_fit_decreasing"
    GREEDY_KNAPSACK = "greedy_knapsack"
    BALANCED_GREEDY_KNAPSACK = "balanced_greedy_knapsack"


class SequencePacker:
    """Base packer.  ``min_bin_count`` / ``bin_count_multiple`` make the bin
    count at least / a multiple of the given number (data-parallel ranks each
    need a micro-batch, and the same number of them); ``max_sequences_per_bin``
    caps the items per bin."""

    def __init__(self, bin_capacity: int, collect_metrics: bool = False, min_bin_count: Optional[int] = None,
                 bin_count_multiple: Optional[int] = None, max_sequences_per_bin: Optional[int] = None,
                 seed: int = 0):
        if bin_capacity <= 0:
            raise ValueError("bin_capacity must be positive")
        if min_bin_count is not None and min_bin_count < 0:
            raise ValueError("min_bin_count must be nonnegative")
        if bin_count_multiple is not None and bin_count_multiple < 1:
            raise ValueError("bin_count_multiple must be positive")
        if max_sequences_per_bin is not None and max_sequences_per_bin < 1:
            raise ValueError("max_sequences_per_bin must be >= 1 (or None for unlimited)")
        self.bin_capacity = int(bin_capacity)
        self.collect_metrics = collect_metrics
        self.min_bin_count = min_bin_count
        self.bin_count_multiple = bin_count_multiple
        self.max_sequences_per_bin = max_sequences_per_bin
        self.seed = seed
        self.last_metrics: dict = {}

    def _fits(self, count: int) -> bool:
        """Room for one more item in a bin that holds ``count``."""
        return self.max_sequences_per_bin is None or count < self.max_sequences_per_bin

    def _pack(self, lengths: list[int]) -> list[list[int]]:
        raise NotImplementedError

    def pack(self, sequence_lengths: list[int]) -> list[list[int]]:
        lengths = [int(x) for x in sequence_lengths]
        for L in lengths:
            if L <= 0:
                raise ValueError("sequence lengths must be positive")
            if L > self.bin_capacity:
                raise ValueError(f"sequence of length {L} exceeds bin capacity {self.bin_capacity}")
        if not lengths:
            return []
        bins = [b for b in self._pack(lengths) if b]
        bins = self._adjust_bin_count(bins, lengths)
        if self.collect_metrics:
            used = [sum(lengths[i] for i in b) for b in bins]
            self.last_metrics = {
                "num_bins": len(bins),
                "utilization": sum(used) / (len(bins) * self.bin_capacity),
                "max_bin_tokens": max(used),
                "min_bin_tokens": min(used),
            }
        return bins

    def _adjust_bin_count(self, bins: list[list[int]], lengths: list[int]) -> list[list[int]]:
        target = len(bins)
        if self.min_bin_count is not None:
            target = max(target, self.min_bin_count)
        if self.bin_count_multiple is not None and target % self.bin_count_multiple:
            target += self.bin_count_multiple - target % self.bin_count_multiple
        if target == len(bins):
            return bins
        if len(lengths) < target:
            raise ValueError(f"Cannot create {target} bins with only {len(lengths)} sequences: every bin needs "
                             "one; lower min_bin_count / bin_count_multiple or pass more sequences")
        return _split_to_min_bins(bins, lengths, target)


def _split_to_min_bins(bins: list[list[int]], lengths: list[int], min_bins: int) -> list[list[int]]:
    """Split the fullest multi-item bins in two (halves of about equal tokens)
    until ``min_bins`` bins exist; the halves keep every bin within capacity
    and within the item cap, and the rest of the packing is untouched."""
    bins = [list(b) for b in bins]
    while len(bins) < min_bins:
        cands = [b for b in bins if len(b) > 1]
        if not cands:
            break
        b = max(cands, key=lambda bb: sum(lengths[i] for i in bb))
        bins.remove(b)
        order = sorted(b, key=lambda i: -lengths[i])
        left, right, lt, rt = [], [], 0, 0
        for i in order:
            if lt <= rt:
                left.append(i)
                lt += lengths[i]
            else:
                right.append(i)
                rt += lengths[i]
        bins += [left, right]
    return bins


class ConcatenativePacker(SequencePacker):
    """Fill bins in input order, opening a new bin when the next item does not fit."""

    def _pack(self, lengths):
        bins, cur, used = [], [], 0
        for i, L in enumerate(lengths):
            if used + L > self.bin_capacity or not self._fits(len(cur)):
                bins.append(cur)
                cur, used = [], 0
            cur.append(i)
            used += L
        bins.append(cur)
        return bins


class FirstFitPacker(SequencePacker):
    def _order(self, lengths: list[int]) -> list[int]:
        return list(range(len(lengths)))

    def _pack(self, lengths):
        bins: list[list[int]] = []
        free: list[int] = []
        for i in self._order(lengths):
            L = lengths[i]
            for b, room in enumerate(free):
                if room >= L and self._fits(len(bins[b])):
                    bins[b].append(i)
                    free[b] -= L
                    break
            else:
                bins.append([i])
                free.append(self.bin_capacity - L)
        return bins


class FirstFitDecreasingPacker(FirstFitPacker):
    def _order(self, lengths):
        return sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))


class FirstFitShufflePacker(FirstFitPacker):
    def _order(self, lengths):
        order = list(range(len(lengths)))
        random.Random(self.seed).shuffle(order)
        return order


class ModifiedFirstFitDecreasingPacker(SequencePacker):
    def _pack(self, lengths):
        if self.max_sequences_per_bin is not None:
            # The class phases only reason about token room; with an item cap
            # first-fit-decreasing (which checks both) packs instead.
            return FirstFitDecreasingPacker(self.bin_capacity, max_sequences_per_bin=self.max_sequences_per_bin
                                            )._pack(lengths)
        C = self.bin_capacity
        idx = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
        large = [i for i in idx if lengths[i] > C / 2]
        medium = [i for i in idx if C / 3 < lengths[i] <= C / 2]
        small = [i for i in idx if C / 6 < lengths[i] <= C / 3]
        tiny = [i for i in idx if lengths[i] <= C / 6]

        bins = [[i] for i in large]
        room = [C - lengths[i] for i in large]
        has_medium = [False] * len(bins)

        # Medium items into large bins: largest remaining medium that fits each bin,
        # visiting bins from the largest item down.
        remaining_medium = list(medium)
        for b in range(len(bins)):
            for j, m in enumerate(remaining_medium):
                if lengths[m] <= room[b]:
                    bins[b].append(m)
                    room[b] -= lengths[m]
                    has_medium[b] = True
                    remaining_medium.pop(j)
                    break

        # Pairs of small items into bins without a medium item, visiting bins from
        # the one with the least room: the smallest small item plus the largest
        # small item that still fits with it.
        remaining_small = list(small)  # sorted decreasing
        for b in sorted(range(len(bins)), key=lambda bb: room[bb]):
            if has_medium[b] or len(remaining_small) < 2:
                continue
            smallest = remaining_small[-1]
            if lengths[smallest] > room[b]:
                continue
            partner = None
            for j in range(len(remaining_small) - 1):
                cand = remaining_small[j]
                if lengths[cand] + lengths[smallest] <= room[b]:
                    partner = j
                    break
            if partner is None:
                continue
            cand = remaining_small.pop(partner)
            remaining_small.pop()  # smallest
            bins[b] += [cand, smallest]
            room[b] -= lengths[cand] + lengths[smallest]

        # Everything left: first-fit-decreasing over existing bins, then new bins.
        leftovers = sorted(remaining_medium + remaining_small + tiny, key=lambda i: (-lengths[i], i))
        for i in leftovers:
            L = lengths[i]
            for b in range(len(bins)):
                if room[b] >= L:
                    bins[b].append(i)
                    room[b] -= L
                    break
            else:
                bins.append([i])
                room.append(C - L)
        return bins


class GreedyKnapsackPacker(SequencePacker):
    """Fill one bin at a time with the largest remaining item that fits."""

    def _pack(self, lengths):
        remaining = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
        bins = []
        while remaining:
            room = self.bin_capacity
            cur = []
            keep = []
            for i in remaining:
                if lengths[i] <= room and self._fits(len(cur)):
                    cur.append(i)
                    room -= lengths[i]
                else:
                    keep.append(i)
            bins.append(cur)
            remaining = keep
        return bins


class BalancedGreedyKnapsackPacker(SequencePacker):
    """Start from the greedy bin count (plus ``balanced_knapsack_delta`` extra
    bins), then place items largest-first into the least-loaded bin that still
    has room (equalises per-micro-batch work); a pass that cannot place an item
    restarts with one more bin."""

    def __init__(self, bin_capacity: int, *args, balanced_knapsack_delta: int = 0, **kwargs):
        super().__init__(bin_capacity, *args, **kwargs)
        if balanced_knapsack_delta < 0:
            raise ValueError("balanced_knapsack_delta must be nonnegative")
        self.balanced_knapsack_delta = int(balanced_knapsack_delta)

    def _pack(self, lengths):
        greedy = GreedyKnapsackPacker(self.bin_capacity, max_sequences_per_bin=self.max_sequences_per_bin)
        n_bins = len(greedy._pack(lengths)) + self.balanced_knapsack_delta
        if self.min_bin_count:
            n_bins = max(n_bins, self.min_bin_count)
        while True:
            bins = [[] for _ in range(n_bins)]
            load = [0] * n_bins
            ok = True
            for i in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
                order = sorted(range(n_bins), key=lambda b: load[b])
                for b in order:
                    if load[b] + lengths[i] <= self.bin_capacity and self._fits(len(bins[b])):
                        bins[b].append(i)
                        load[b] += lengths[i]
                        break
                else:
                    ok = False
                    break
            if ok:
                return bins
            n_bins += 1


_PACKERS = {
    PackingAlgorithm.CONCATENATIVE: ConcatenativePacker,
    PackingAlgorithm.FIRST_FIT: FirstFitPacker,
    PackingAlgorithm.FIRST_FIT_DECREASING: FirstFitDecreasingPacker,
    PackingAlgorithm.FIRST_FIT_SHUFFLE: FirstFitShufflePacker,
    PackingAlgorithm.MODIFIED_FIRST_FIT_DECREASING: ModifiedFirstFitDecreasingPacker,
    PackingAlgorithm.GREEDY_KNAPSACK: GreedyKnapsackPacker,
    PackingAlgorithm.BALANCED_GREEDY_KNAPSACK: BalancedGreedyKnapsackPacker,
}


def get_packer(algorithm, bin_capacity: int, **kwargs) -> SequencePacker:
    if isinstance(algorithm, str):
        algorithm = PackingAlgorithm(algorithm)
    return _PACKERS[algorithm](bin_capacity, **kwargs)
