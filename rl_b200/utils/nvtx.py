"""NVTX ranges and step-range profiler capture.

Reference: ``wrap_with_nvtx_name`` (``nemo_rl/utils/nsys.py:113``) and
``maybe_gpu_profile_step`` (``:62``, env ``NRL_NSYS_PROFILE_STEP_RANGE``).  Here the
env variable is ``RLB_PROFILE_STEP_RANGE="start:stop"`` (steps, stop exclusive):
``cudaProfilerStart`` / ``Stop`` bracket those steps, so an external profiler
started with ``--capture-range=cudaProfilerApi`` records only them.  Ranges are
no-ops without CUDA.
"""

from __future__ import annotations

import contextlib
import functools
import os

import torch

__all__ = ["nvtx_range", "wrap_with_nvtx_name", "maybe_gpu_profile_step", "profile_step_range"]

_ON = torch.cuda.is_available() and os.environ.get("RLB_NVTX", "1") != "0"


@contextlib.contextmanager
def nvtx_range(name: str):
    if _ON:
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def wrap_with_nvtx_name(name: str):
    def deco(fn):
        @functools.wraps(fn)
        def inner(*a, **k):
            with nvtx_range(name):
                return fn(*a, **k)
        return inner
    return deco


def profile_step_range() -> tuple[int, int] | None:
    v = os.environ.get("RLB_PROFILE_STEP_RANGE")
    if not v:
        return None
    a, b = v.split(":")
    return int(a), int(b)


_active = False


def maybe_gpu_profile_step(step: int) -> None:
    """Call at the start of every step."""
    global _active
    rng = profile_step_range()
    if rng is None or not torch.cuda.is_available():
        return
    start, stop = rng
    if step == start and not _active:
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        _active = True
    elif step == stop and _active:
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        _active = False
