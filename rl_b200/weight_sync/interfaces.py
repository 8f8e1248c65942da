"""Weight-synchronizer interface (train -> rollout refit).

Reference: ``WeightSynchronizer`` (``nemo_rl/weight_sync/interfaces.py:77``) and
``create_weight_synchronizer`` (``nemo_rl/weight_sync/factory.py:79``): one object
owns a transport's lifecycle - set up once, then ``sync`` after every optimizer
step, ``shutdown`` at the end.  Transports here:

* ``inplace``   - colocated, same layout: the rollout engine reads the trainer's
  bf16 parameters, nothing moves (``ColocatedInPlaceSynchronizer``);
* ``reshard``   - colocated, different TP layout and / or fp8 rollout weights:
  one native kernel per rank loads the training shards from the TP peers'
  HBM over NVLink and writes the generation layout, fused with the bf16 copy
  or the 128x128 e4m3 quantisation (``ColocatedReshardSynchronizer``);
* ``broadcast`` - non-colocated trainer / generation processes: packed,
  double-buffered bucket broadcast over a (stateless) process group
  (``PackedBroadcastSynchronizer``);
* ``sparse_broadcast`` - the same transport sending, after a first full refit,
  only the weights whose bits changed (``SparseDeltaBroadcastSynchronizer``).

``create_weight_synchronizer(kind, **kwargs)`` builds one by name (the
reference's ``refit_transport`` values map onto these).
"""

from __future__ import annotations

import abc
import time
from typing import Any

__all__ = ["WeightSynchronizer"]


class WeightSynchronizer(abc.ABC):
    name = "base"

    def __init__(self):
        self.version = 0
        self.stats: dict[str, Any] = {"syncs": 0, "last_s": 0.0, "bytes": 0}

    def prepare(self) -> None:
        """One-time set-up (buffers, plans, communicators)."""

    @abc.abstractmethod
    def _sync(self) -> int:
        """Move the weights; returns the bytes written on this rank."""

    def sync(self) -> dict:
        t0 = time.perf_counter()
        nbytes = self._sync()
        self.version += 1
        self.stats["syncs"] += 1
        self.stats["last_s"] = time.perf_counter() - t0
        self.stats["bytes"] = int(nbytes)
        return dict(self.stats, version=self.version)

    def shutdown(self) -> None:
        """Release buffers / communicators (idempotent)."""
