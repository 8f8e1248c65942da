"""NVLink SHARP buffers: NVSwitch multicast memory with this package's multimem
kernels (``csrc/nvls.cu``).

The allocation and the multicast binding come from PyTorch's symmetric memory
(``torch.distributed._symmetric_memory``: ``empty`` + ``rendezvous`` give every
rank's buffer address, a multicast address when the driver and switch support
it, and per-rank signal words).  The collectives themselves are this package's
kernels: ``multimem.ld_reduce`` reads the sum of all ranks' values through the
switch, ``multimem.st`` writes one value to every rank, and a bounded
signal-word barrier orders the ranks around each call.

``NVLSBuffer.all_reduce_()`` sums the buffer over the group in place;
``reduce_shard(lo, n, out)`` sums a range into a local tensor (each rank asking
for its own shard is a reduce-scatter).  Reference counterpart: the NVLS
collectives NCCL runs for MCore on NVSwitch systems.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from rl_b200.ops._ext import ext

__all__ = ["NVLSBuffer"]


def _symm():
    import torch.distributed._symmetric_memory as symm_mem

    return symm_mem


def _group_name(group) -> str:
    g = group if group is not None else dist.group.WORLD
    return g.group_name


class NVLSBuffer:
    """``numel`` elements of ``dtype`` (fp32 or bf16) bound to a multicast object
    over ``group`` (collective: every rank of the group constructs it)."""

    def __init__(self, numel: int, dtype: torch.dtype, group=None, device: Optional[torch.device] = None):
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("NVLSBuffer holds fp32 or bf16")
        sm = _symm()
        self.group = group
        name = _group_name(group)
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.tensor = sm.empty(numel, dtype=dtype, device=device)
        self.handle = sm.rendezvous(self.tensor, name)
        self.mc_ptr = int(self.handle.multicast_ptr or 0)  # 0 when the system has no multicast support
        if not self.mc_ptr:
            raise RuntimeError("NVLS multicast is not available on this system (no multicast address)")
        self.rank, self.world = int(self.handle.rank), int(self.handle.world_size)
        # signal words: the upper half of every rank's pad (the lower half is left to PyTorch)
        words = int(self.handle.signal_pad_size) // 4
        self._pads = [int(p) + 4 * (words // 2) for p in self.handle.signal_pad_ptrs]
        if words // 2 < self.world:
            raise RuntimeError("signal pad too small for the group")
        self.epoch = 0
        self.f32 = dtype == torch.float32

    def barrier(self) -> None:
        self.epoch += 1
        ext().nvls_barrier(self._pads, self.rank, self.epoch)

    def all_reduce_(self) -> torch.Tensor:
        """Sum ``self.tensor`` over the group in place (barrier, multimem reduce +
        store of this rank's slice, barrier)."""
        nbytes = self.tensor.numel() * self.tensor.element_size()
        self.barrier()
        ext().nvls_all_reduce(self.mc_ptr, nbytes, self.f32, self.rank, self.world)
        self.barrier()
        return self.tensor

    def reduce_shard(self, lo: int, n: int, out: torch.Tensor) -> torch.Tensor:
        """``out[:] = sum over ranks of tensor[lo:lo + n]`` (elements)."""
        es = self.tensor.element_size()
        self.barrier()
        ext().nvls_reduce_shard(self.mc_ptr, lo * es, n * es, out, self.f32)
        self.barrier()
        return out
