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

__all__ = ["PackedBroadcastSynchronizer", "SparseDeltaBroadcastSynchronizer", "bucket_bytes_for"]


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


class SparseDeltaBroadcastSynchronizer(PackedBroadcastSynchronizer):
    """Non-colocated refit that sends only the weights whose stored bits changed
    since the last refit.

    Reference: the sparse remote refit transports (``vllm_s3_sparse`` /
    ``vllm_zmq_sparse``, ``nemo_rl/weight_sync/vllm_remote_sparse_weight_synchronizer.py``).
    At RL learning rates most bf16 weights keep their exact bits from one step
    to the next (an update smaller than half a unit in the last place of the
    weight does not change it), so the changed set is a small fraction of the
    model.  The producer keeps a copy of what it last sent; per bucket it
    compares raw bits, then broadcasts a header (mode, count) followed either by
    the int32 positions and values of the changed elements, or by the whole
    bucket when more than ``dense_fraction`` of it changed (positions would cost
    more than they save).  Consumers apply the scatter into their flat buffer.
    The first refit (and every ``full_every``-th, if set) sends everything.
    ``sync()["bytes"]`` reports what actually crossed the wire."""
    name = "sparse_broadcast"

    def __init__(self, flat: torch.Tensor, group, src: int = 0, bucket_bytes: Optional[int] = None,
                 timeout_s: float = 600.0, dense_fraction: float = 0.25, full_every: int = 0):
        super().__init__(flat, group, src, bucket_bytes, timeout_s)
        self.dense_fraction = float(dense_fraction)
        self.full_every = int(full_every)
        self.syncs = 0
        self.sent: Optional[torch.Tensor] = None  # producer: the last transmitted version
        self.last_stats: dict = {}

    def _bits(self, t: torch.Tensor) -> torch.Tensor:
        view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
        return t.view(view)

    def _sync(self) -> int:
        hold_refit_for_fault_injection()
        n = self.flat.numel()
        producer = self.group.rank == self.src
        full = self.syncs == 0 or (self.full_every > 0 and self.syncs % self.full_every == 0)
        self.syncs += 1
        dev = self.flat.device
        moved, changed = 0, 0
        with RefitAbortWatchdog(self.timeout_s, self.group.abort) as wd:
            if full:
                for lo in range(0, n, self.bucket_elems):
                    self.group.broadcast(self.flat[lo: lo + self.bucket_elems], self.src)
                moved = n * self.flat.element_size()
                changed = n
                if producer:
                    self.sent = self.flat.detach().clone()
            else:
                for lo in range(0, n, self.bucket_elems):
                    hi = min(n, lo + self.bucket_elems)
                    cur = self.flat[lo:hi]
                    hdr = torch.zeros(2, dtype=torch.int64, device=dev)
                    if producer:
                        idx = torch.nonzero(self._bits(cur) != self._bits(self.sent[lo:hi])).flatten()
                        dense = idx.numel() > self.dense_fraction * (hi - lo)
                        hdr[0], hdr[1] = (1 if dense else 0), idx.numel()
                    self.group.broadcast(hdr, self.src)
                    mode, cnt = int(hdr[0]), int(hdr[1])
                    moved += hdr.numel() * hdr.element_size()
                    changed += cnt
                    if cnt == 0:
                        continue
                    if mode == 1:
                        self.group.broadcast(cur, self.src)
                        moved += cur.numel() * cur.element_size()
                    else:
                        pos = idx.to(torch.int32) if producer else torch.empty(cnt, dtype=torch.int32, device=dev)
                        vals = cur[idx] if producer else torch.empty(cnt, dtype=cur.dtype, device=dev)
                        self.group.broadcast(pos, self.src)
                        self.group.broadcast(vals, self.src)
                        moved += cnt * (4 + cur.element_size())
                        if not producer:
                            cur[pos.long()] = vals
                    if producer:
                        self.sent[lo:hi].copy_(cur)
        self.aborted = wd.fired
        self.last_stats = {"changed_elements": changed, "changed_fraction": changed / max(1, n),
                           "full": float(full)}
        return moved
