"""Loader for the in-tree native extension ``rl_b200._C`` (sm_100a kernels).

CPU tensors always take the PyTorch reference path (the fp32 oracle used by
tests and by the CPU plumbing run).  CUDA tensors MUST take the native path: if
the extension is missing on a GPU box the op raises instead of silently
falling back, so a run never reports numbers from a fallback by accident.

Every call into the extension goes through a counting proxy: ``launch_count()``
returns how many native kernels have been launched (each entry point adds the
number of kernels it launches; CUDA-graph replays add the count recorded at
capture).  Benchmarks report this as their native launch count.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

_EXT: Optional[Any] = None
_ERR: Optional[BaseException] = None
_LAUNCHES = 0
_CAPTURE_DEPTH = 0

# kernels launched per entry-point call (default 1)
_KERNELS_PER_CALL = {
    "rmsnorm_bwd": 2,
    "rmsnorm_bwd_add": 2,
    "sum_sq": 2,
    "flash_attn_bwd": 3,
    "flash_attn_seg_bwd": 3,
    "flash_attn_bwd_tc": 3,
    "flash_attn_seg_bwd_tc": 3,
    "paged_decode_attn": 1,
    "sample": 2,
    "gemm_error_flag": 0,
    "gemm_fp8_error_flag": 0,
    "grouped_gemm_error_flag": 0,
    "gemm_decode_error_flag": 0,
    "stream_write_u32": 0,
    "decode_ar_error_flag": 0,
    "attn_error_flag": 0,
    "ep_error_flag": 0,
    "gemm_sm100_error_flag": 0,
    "attn_tc_error_flag": 0,
    "peer_wait_cycles": 0,
    "set_peer_wait_cycles": 0,
    "symm_alloc": 0,
    "symm_open": 0,
    "symm_close": 0,
    "symm_view": 0,
    "moe_router_topk": 3,
    "bounds_errors": 0,
    "dp_error_flag": 0,
    "nvls_error_flag": 0,
    "debug_bounds_build": 0,
}


class _Counting:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        n = _KERNELS_PER_CALL.get(name, 1)

        def wrapped(*a, **k):
            global _LAUNCHES
            _LAUNCHES += n
            return fn(*a, **k)

        return wrapped


def _load():
    global _EXT, _ERR
    if _EXT is not None or _ERR is not None:
        return
    try:
        import os

        if os.environ.get("RL_B200_DEBUG_BOUNDS", "0") == "1":
            # bounds-checked debug build (setup.py with RL_B200_DEBUG_BOUNDS=1)
            from rl_b200 import _C_debug as _C  # type: ignore
        else:
            from rl_b200 import _C  # type: ignore

        _EXT = _Counting(_C)
    except BaseException as e:  # noqa: BLE001 - record and re-raise at use
        _ERR = e


def has_ext() -> bool:
    _load()
    return _EXT is not None


def ext():
    """Return the native module, raising a clear error when it is unavailable."""
    _load()
    if _EXT is None:
        raise RuntimeError(
            "rl_b200 native extension (rl_b200/_C*.so) is not built or failed to load: "
            f"{_ERR!r}. Build it with `python setup.py build_ext --inplace` "
            "(or __graft_entry__.build())."
        )
    return _EXT


def launch_count() -> int:
    return _LAUNCHES


def add_launches(n: int) -> None:
    """Account kernels launched outside a direct call (CUDA-graph replays)."""
    global _LAUNCHES
    _LAUNCHES += n


def use_native(*tensors: torch.Tensor) -> bool:
    """True when the op must run on the native CUDA path."""
    return any(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors)


# every kernel family's device error word (set when a bounded wait runs out)
ERROR_FLAGS = ("gemm_error_flag", "gemm_sm100_error_flag", "gemm_fp8_error_flag", "grouped_gemm_error_flag",
               "gemm_decode_error_flag", "decode_ar_error_flag", "attn_error_flag", "attn_tc_error_flag",
               "ep_error_flag", "dp_error_flag", "nvls_error_flag")


BOUNDS_SITES = {1: "KV-cache slot", 2: "paged-attention block-table entry",
                3: "expert-parallel row / rank", 4: "MoE router expert-grouped row"}


class DeviceBoundsError(RuntimeError):
    """The bounds-checked debug build met a data-dependent index outside its
    tensor (the access was skipped)."""


class DeviceWaitError(RuntimeError):
    """A kernel gave up a bounded wait (a peer's flag, a copy engine's flag or a
    pipeline barrier never arrived) and returned with its error word set."""


def check_device_errors(reset: bool = True) -> None:
    """Read (and by default clear) every kernel family's error word; raise
    :class:`DeviceWaitError` naming the ones that are set.  One small device read
    per family: callers run it at step boundaries, not per kernel."""
    if not has_ext():
        return
    mod = ext()
    bad = {}
    for name in ERROR_FLAGS:
        fn = getattr(mod, name, None)
        if fn is None:
            continue
        v = int(fn(reset))
        if v:
            bad[name] = v
    if bad:
        raise DeviceWaitError(f"device wait expired: {bad} (error word = wait site code); "
                              "a peer rank, copy engine or pipeline stage never signalled")
    if getattr(mod, "debug_bounds_build", None) is not None and mod.debug_bounds_build():
        hits = {f: v for f, v in mod.bounds_errors(reset).items() if v}
        if hits:
            raise DeviceBoundsError("index out of bounds (access skipped): " + ", ".join(
                f"{f}: {BOUNDS_SITES.get(v >> 40, v >> 40)} index {v & ((1 << 40) - 1)}" for f, v in hits.items()))
    from rl_b200.parallel.symm import check_canaries

    check_canaries()
