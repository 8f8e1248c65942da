"""Local multi-process launcher: run a function on N ranks of one host.

Used by the distributed tests (gloo ranks on CPU, NCCL ranks on GPUs) and by
users who want SPMD workers without torchrun - the counterpart of the
reference's ``distributed_test_runner`` fixture (``tests/unit/conftest.py:452-535``,
``mp.spawn`` + ``init_process_group`` on localhost).  Each rank gets the torchrun
environment (``RANK``, ``LOCAL_RANK``, ``WORLD_SIZE``, ``MASTER_ADDR=127.0.0.1``,
``MASTER_PORT``) before ``fn(rank, *args)`` runs; return values come back in rank
order, and an exception on any rank is re-raised in the caller.
"""

from __future__ import annotations

import os
import socket
import traceback
from typing import Any, Callable

import torch.multiprocessing as mp

__all__ = ["free_port", "spawn_ranks"]


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Arr:
    """Tensor shipped by value (numpy) so it outlives the producing process."""

    def __init__(self, t):
        self.a = t.detach().cpu().numpy()


def _pack(x):
    import torch

    if isinstance(x, torch.Tensor):
        return _Arr(x)
    if isinstance(x, dict):
        return {k: _pack(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_pack(v) for v in x)
    return x


def _unpack(x):
    import torch

    if isinstance(x, _Arr):
        return torch.from_numpy(x.a)
    if isinstance(x, dict):
        return {k: _unpack(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_unpack(v) for v in x)
    return x


def _entry(rank: int, world: int, port: int, fn: Callable, args: tuple, q) -> None:
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        out = fn(rank, *args)
        q.put((rank, "ok", _pack(out)))
    except BaseException as e:  # noqa: BLE001 - report to the parent
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        try:
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def spawn_ranks(fn: Callable, world: int, *args: Any, timeout_s: float = 300.0) -> list:
    """Run ``fn(rank, *args)`` on ``world`` processes; returns the per-rank results."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q), daemon=False) for r in range(world)]
    for p in procs:
        p.start()
    results: dict[int, Any] = {}
    errors = []
    try:
        for _ in range(world):
            rank, status, val = q.get(timeout=timeout_s)
            if status == "ok":
                results[rank] = _unpack(val)
            else:
                errors.append((rank, val))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    if errors:
        raise RuntimeError("rank failure(s):\n" + "\n".join(f"[rank {r}] {m}" for r, m in errors))
    return [results[r] for r in range(world)]
