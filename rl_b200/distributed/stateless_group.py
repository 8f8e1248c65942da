"""Process groups outside the default ``torch.distributed`` world.

Reference: ``StatelessProcessGroup`` (``nemo_rl/distributed/stateless_process_group.py:91``,
TCPStore + nccl4py, ``abort`` at ``:115``): the refit path between a training world
and separately launched generation processes needs a communicator whose members
belong to different worlds, which can be torn down (aborted) when a peer hangs.

Here the group is a ``TCPStore`` (rank 0 hosts it) plus a ``PrefixStore`` per
group name, and a backend object constructed directly on that store
(``ProcessGroupNCCL`` on CUDA, ``ProcessGroupGloo`` otherwise).  Collectives are
issued asynchronously and waited on with ``wait`` which polls, so a watchdog
(or the caller) can abort a stuck operation: the waiter raises ``GroupAborted``
and, for NCCL, the communicator is aborted so that its kernels return.
"""

from __future__ import annotations

import datetime
import threading
import time
from typing import Optional

import torch
import torch.distributed as dist

__all__ = ["StatelessProcessGroup", "GroupAborted"]


class GroupAborted(RuntimeError):
    pass


class StatelessProcessGroup:
    def __init__(self, host: str, port: int, rank: int, world_size: int, backend: Optional[str] = None,
                 name: str = "stateless", timeout_s: float = 120.0, device: Optional[torch.device] = None):
        self.rank, self.world_size = int(rank), int(world_size)
        self.backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        self.device = device or (torch.device("cuda", torch.cuda.current_device()) if self.backend == "nccl"
                                 else torch.device("cpu"))
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.store = dist.TCPStore(host, int(port), self.world_size, is_master=(self.rank == 0),
                                   timeout=self.timeout, wait_for_workers=True)
        self._prefix = dist.PrefixStore(name, self.store)
        if self.backend == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            self.pg = dist.ProcessGroupNCCL(self._prefix, self.rank, self.world_size, opts)
        else:
            self.pg = dist.ProcessGroupGloo(self._prefix, self.rank, self.world_size, self.timeout)
        self._aborted = threading.Event()

    # ----------------------------------------------------------- collectives
    def _wait(self, work, deadline_s: Optional[float] = None) -> None:
        t_end = time.monotonic() + (deadline_s if deadline_s is not None else self.timeout.total_seconds())
        while not work.is_completed():
            if self._aborted.is_set():
                raise GroupAborted("process group aborted while a collective was pending")
            if time.monotonic() > t_end:
                self.abort()
                raise GroupAborted("collective timed out")
            time.sleep(0.0005)
        work.wait()

    def broadcast(self, t: torch.Tensor, src: int, deadline_s: Optional[float] = None) -> torch.Tensor:
        opts = dist.BroadcastOptions()
        opts.rootRank = int(src)
        opts.rootTensor = 0
        self._wait(self.pg.broadcast([t], opts), deadline_s)
        return t

    def all_reduce(self, t: torch.Tensor, deadline_s: Optional[float] = None) -> torch.Tensor:
        opts = dist.AllreduceOptions()
        opts.reduceOp = dist.ReduceOp.SUM
        self._wait(self.pg.allreduce([t], opts), deadline_s)
        return t

    def barrier(self, deadline_s: Optional[float] = None) -> None:
        x = torch.zeros(1, device=self.device)
        self.all_reduce(x, deadline_s)

    # ------------------------------------------------------------- lifecycle
    @property
    def aborted(self) -> bool:
        return self._aborted.is_set()

    def abort(self) -> None:
        """Make every pending and future wait on this group fail; NCCL
        communicators are aborted so that in-flight kernels return."""
        self._aborted.set()
        if self.backend == "nccl":
            try:
                self.pg.abort()
            except Exception:  # noqa: BLE001 - best effort; the waiters already fail
                pass

    def destroy(self) -> None:
        if self.backend == "nccl" and not self.aborted:
            try:
                self.pg.shutdown()
            except Exception:  # noqa: BLE001
                pass
        self.pg = None
