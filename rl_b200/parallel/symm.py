"""Symmetric device buffers across the ranks of a process group (one node).

Each rank allocates the same number of bytes (raw cudaMalloc in the native
library), the CUDA IPC handles are exchanged over the group, and every rank
opens every peer's handle.  ``ptrs[r]`` is then a device address through which
this rank's kernels load / store rank r's buffer over NVLink (``ptrs[me]`` is
the local allocation).  This is the substrate of the fused compute+collective
kernels in ``rl_b200.parallel.fused``.
"""

from __future__ import annotations

import os
import weakref

import torch
import torch.distributed as dist

from rl_b200.ops._ext import ext

__all__ = ["SymmetricBuffer", "NodeSymmetric", "canaries_enabled", "check_canaries"]

# Canaries: with RL_B200_CANARIES=1 (or the bounds-checked debug build,
# RL_B200_DEBUG_BOUNDS=1) every symmetric buffer is allocated with a guard of
# GUARD bytes before and after it, filled with PATTERN; ``ptrs`` / ``local_ptr``
# point past the head guard, so kernels see the same buffer.  A peer store (or a
# local one) that runs off either end of a buffer lands in a guard, and
# ``check_canaries`` (run with the device error words at step boundaries) names
# the buffer whose guard changed.
GUARD = 4096
PATTERN = 0xA5
_LIVE: "weakref.WeakSet[SymmetricBuffer]" = weakref.WeakSet()


def canaries_enabled() -> bool:
    return os.environ.get("RL_B200_CANARIES", "0") == "1" or os.environ.get("RL_B200_DEBUG_BOUNDS", "0") == "1"


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None):
        self.nbytes = int(nbytes)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.guard = GUARD if canaries_enabled() else 0
        ptr, handle = ext().symm_alloc(self.nbytes + 2 * self.guard)
        self._bases: list[int] = []  # what the allocator / IPC open returned (closed by close())
        self.local_ptr = int(ptr) + self.guard
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
        else:
            handles = [bytes(handle.numpy().tobytes())]
        self.ptrs: list[int] = []
        for r, h in enumerate(handles):
            base = int(ptr) if r == self.rank else \
                int(ext().symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
            self._bases.append(base)
            self.ptrs.append(base + self.guard)
        self.device = torch.cuda.current_device()
        if self.guard:
            for g in self._guards():
                g.fill_(PATTERN)
            _LIVE.add(self)

    def _guards(self) -> list:
        code = 0  # uint8
        return [ext().symm_view(self.local_ptr - self.guard, self.guard, code, self.device),
                ext().symm_view(self.local_ptr + self.nbytes, self.guard, code, self.device)]

    def canary_intact(self) -> bool:
        """Whether both guards of this rank's buffer still hold the pattern."""
        if not self.guard or not self.ptrs:
            return True
        return all(bool((g == PATTERN).all()) for g in self._guards())

    def local_view(self, dtype: torch.dtype, numel: int, offset_bytes: int = 0) -> torch.Tensor:
        code = {torch.bfloat16: 15, torch.float32: 6, torch.int32: 3, torch.uint8: 0}[dtype]
        return ext().symm_view(self.local_ptr + offset_bytes, numel, code, self.device)

    def close(self) -> None:
        for r, p in enumerate(self._bases):
            if r != self.rank:
                ext().symm_close(p)
        if self._bases:
            ext().symm_close(self._bases[self.rank])
        self.ptrs, self._bases = [], []
        _LIVE.discard(self)

    def close_collective(self) -> None:
        """Collective release: every rank unmaps its peers' buffers, all ranks
        synchronise, then each frees its own allocation (no rank frees memory a
        peer still maps)."""
        for r, p in enumerate(self._bases):
            if r != self.rank:
                ext().symm_close(p)
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        if self._bases:
            ext().symm_close(self._bases[self.rank])
        self.ptrs, self._bases = [], []
        _LIVE.discard(self)


def check_canaries() -> None:
    """Raise ``DeviceBoundsError`` when a guard of a live symmetric buffer of this
    rank was overwritten (canaries on); no-op otherwise."""
    if not _LIVE:
        return
    from rl_b200.ops._ext import DeviceBoundsError

    bad = [b for b in list(_LIVE) if not b.canary_intact()]
    if bad:
        raise DeviceBoundsError("symmetric buffer guard overwritten (a store ran off a buffer's end): " +
                                ", ".join(f"{b.nbytes} B buffer at 0x{b.local_ptr:x}" for b in bad))


class NodeSymmetric:
    """Allocator of symmetric buffers across every rank of a single-node job
    (``group`` defaults to the world): ``ptrs`` are indexed by the group rank,
    which for the world group is the global rank, so TP, DP and EP peers are
    all addressable.  ``flat_alloc`` is the ``TransformerLM`` flat-buffer hook: the
    returned tensor carries its ``SymmetricBuffer`` as ``tensor._symm``."""

    def __init__(self, group=None):
        self.group = group
        self.buffers: list[SymmetricBuffer] = []

    def alloc(self, nbytes: int) -> SymmetricBuffer:
        b = SymmetricBuffer(nbytes, self.group)
        self.buffers.append(b)
        return b

    def flat_alloc(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        elt = torch.empty((), dtype=dtype).element_size()
        b = self.alloc(numel * elt)
        t = b.local_view(dtype, numel)
        t._symm = b
        return t

    def release(self, buf: SymmetricBuffer) -> None:
        if buf in self.buffers:
            self.buffers.remove(buf)
            buf.close_collective()

    @staticmethod
    def supported() -> bool:
        """CUDA, initialised process group, every rank on this node."""
        import os

        if not (torch.cuda.is_available() and dist.is_initialized()):
            return False
        world = dist.get_world_size()
        local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
        return world > 1 and local == world
