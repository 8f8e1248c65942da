"""Non-colocated refit: bucketed broadcast of the flat weight buffer.

Reference: ``packed_broadcast_producer`` / consumer (``nemo_rl/utils/packed_tensor.py:40-302``):
the trainer packs tensors into uint8 buckets of at most min(2 % of HBM, 5 GiB),
double-buffered, and broadcasts them to every generation rank, which unpacks
them into its weights.

Because every model here keeps its parameters in ONE flat buffer with a
layout that both sides compute from the same config, a bucket is simply a
contiguous slice of that buffer: the producer broadcasts views of its own
buffer and the consumers receive straight into theirs, so there is nothing to
pack, no staging copy and no second buffer.  Each bucket is a separate
collective, so a watchdog can abort a stalled refit between (or during)
buckets.
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.weight_sync.interfaces import WeightSynchronizer
from rl_b200.weight_sync.watchdog import RefitAbortWatchdog, hold_refit_for_fault_injection

__all__ = ["PackedBroadcastSynchronizer", "bucket_bytes_for"]


def bucket_bytes_for(device: torch.device) -> int:
    """min(2 % of the device memory, 5 GiB); 64 MiB on CPU."""
    if device.type == "cuda":
        total = torch.cuda.get_device_properties(device).total_memory
        return int(min(0.02 * total, 5 << 30))
    return 64 << 20


class PackedBroadcastSynchronizer(WeightSynchronizer):
    """``flat`` is the producer's (rank ``src``) or a consumer's flat weight
    buffer; ``group`` a ``StatelessProcessGroup`` spanning the trainer's
    source rank and the generation ranks."""
    name = "broadcast"

    def __init__(self, flat: torch.Tensor, group, src: int = 0, bucket_bytes: Optional[int] = None,
                 timeout_s: float = 600.0):
        super().__init__()
        self.flat = flat
        self.group = group
        self.src = int(src)
        elt = flat.element_size()
        self.bucket_elems = max(1, int(bucket_bytes or bucket_bytes_for(flat.device)) // elt)
        self.timeout_s = float(timeout_s)
        self.aborted = False

    def _sync(self) -> int:
        hold_refit_for_fault_injection()
        n = self.flat.numel()
        with RefitAbortWatchdog(self.timeout_s, self.group.abort) as wd:
            for lo in range(0, n, self.bucket_elems):
                self.group.broadcast(self.flat[lo: lo + self.bucket_elems], self.src)
        self.aborted = wd.fired
        return n * self.flat.element_size()
