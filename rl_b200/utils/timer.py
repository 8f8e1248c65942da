"""Named timers (host wall clock and CUDA-event device time) and a deadline checker.

Reference: ``Timer`` (``nemo_rl/utils/timer.py:29``) feeding the ``timing/*`` metrics
and ``TimeoutChecker`` (``:439``) used with ``checkpoint_must_save_by``.
``DeviceTimer`` adds CUDA-event timing (time on the launching stream, taken
after a synchronize) and a max-over-ranks reduction for multi-GPU numbers.
"""

from __future__ import annotations

import contextlib
import time
from collections import defaultdict
from typing import Optional

import torch
import torch.distributed as dist

__all__ = ["Timer", "DeviceTimer", "TimeoutChecker", "max_over_ranks"]


class Timer:
    def __init__(self):
        self._start: dict[str, float] = {}
        self._times: dict[str, list[float]] = defaultdict(list)

    def start(self, label: str) -> None:
        if label in self._start:
            raise RuntimeError(f"timer {label!r} already running")
        self._start[label] = time.perf_counter()

    def stop(self, label: str) -> float:
        if label not in self._start:
            raise RuntimeError(f"timer {label!r} was not started")
        dt = time.perf_counter() - self._start.pop(label)
        self._times[label].append(dt)
        return dt

    @contextlib.contextmanager
    def time(self, label: str):
        """Time a block (host wall clock) and mark it as an NVTX range."""
        from rl_b200.utils.nvtx import nvtx_range

        self.start(label)
        try:
            with nvtx_range(label):
                yield
        finally:
            self.stop(label)

    def get_elapsed(self, label: str, reduction: str = "sum") -> float:
        v = self._times.get(label, [])
        if not v:
            return 0.0
        if reduction == "sum":
            return float(sum(v))
        if reduction == "mean":
            return float(sum(v) / len(v))
        if reduction == "max":
            return float(max(v))
        if reduction == "min":
            return float(min(v))
        if reduction == "last":
            return float(v[-1])
        raise ValueError(reduction)

    def get_timing_metrics(self, reduction_op: str = "sum") -> dict[str, float]:
        return {k: self.get_elapsed(k, reduction_op) for k in self._times}

    def reset(self, label: Optional[str] = None) -> None:
        if label is None:
            self._times.clear()
            self._start.clear()
        else:
            self._times.pop(label, None)
            self._start.pop(label, None)


class DeviceTimer:
    """CUDA-event interval timer on the current stream (ms)."""

    def __init__(self):
        self.cuda = torch.cuda.is_available()

    @contextlib.contextmanager
    def time(self, out: dict, label: str):
        if not self.cuda:
            t0 = time.perf_counter()
            yield
            out[label] = out.get(label, 0.0) + (time.perf_counter() - t0) * 1e3
            return
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        yield
        b.record()
        torch.cuda.synchronize()
        out[label] = out.get(label, 0.0) + a.elapsed_time(b)


def max_over_ranks(value: float, group=None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() and \
        dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class TimeoutChecker:
    """Tracks iteration durations and reports when the next iteration would cross a
    wall-clock deadline (``checkpoint_must_save_by`` = "DD:HH:MM:SS" from start)."""

    def __init__(self, timeout: Optional[str] = None, fit_last_save_time: bool = True):
        self.start = time.time()
        self.deadline = None
        if timeout:
            parts = [int(x) for x in str(timeout).split(":")]
            while len(parts) < 4:
                parts.insert(0, 0)
            d, h, m, s = parts
            self.deadline = self.start + d * 86400 + h * 3600 + m * 60 + s
        self.fit_last = fit_last_save_time
        self.iter_times: list[float] = []
        self._last = None

    def start_iterations(self) -> None:
        self._last = time.time()

    def mark_iteration(self) -> None:
        now = time.time()
        if self._last is not None:
            self.iter_times.append(now - self._last)
        self._last = now

    def check_save(self) -> bool:
        if self.deadline is None:
            return False
        nxt = max(self.iter_times) if (self.iter_times and self.fit_last) else 0.0
        return time.time() + nxt >= self.deadline
