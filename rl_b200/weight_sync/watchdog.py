"""Refit watchdog and host-side fault injection.

Reference: ``RefitAbortWatchdog`` (``nemo_rl/distributed/refit_watchdog.py:309``)
aborts a hung refit communicator after a deadline, and
``hold_refit_for_fault_injection`` (``:476``) holds a refit while a file exists
so that tests can simulate a stuck peer.

``RefitAbortWatchdog`` is a context manager: if the guarded block has not
finished within ``timeout_s`` its ``on_abort`` callback runs (typically
``StatelessProcessGroup.abort``), ``fired`` is set, and the block's pending
collective fails with ``GroupAborted``.  Fault injection is host-side only: a
rank is held (sleeping on the host, no kernel in flight) while the hold file
exists, so no GPU is ever made to hang.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Callable, Optional

__all__ = ["RefitAbortWatchdog", "hold_refit_for_fault_injection", "HOLD_FILE_ENV"]

HOLD_FILE_ENV = "RLB_REFIT_HOLD_FILE"


class RefitAbortWatchdog:
    def __init__(self, timeout_s: float, on_abort: Callable[[], None], name: str = "refit"):
        self.timeout_s = float(timeout_s)
        self.on_abort = on_abort
        self.name = name
        self.fired = False
        self._done = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.elapsed_s = 0.0

    def _run(self, t0: float) -> None:
        if not self._done.wait(self.timeout_s):
            self.fired = True
            try:
                self.on_abort()
            finally:
                self.elapsed_s = time.monotonic() - t0

    def __enter__(self) -> "RefitAbortWatchdog":
        self._done.clear()
        self.fired = False
        t0 = time.monotonic()
        self._thread = threading.Thread(target=self._run, args=(t0,), name=f"{self.name}-watchdog", daemon=True)
        self._thread.start()
        self._t0 = t0
        return self

    def __exit__(self, *exc) -> bool:
        self._done.set()
        if self._thread is not None:
            self._thread.join(timeout=max(1.0, self.timeout_s))
        if not self.fired:
            self.elapsed_s = time.monotonic() - self._t0
        return False


def hold_refit_for_fault_injection(max_hold_s: float = 600.0, poll_s: float = 0.05) -> float:
    """If ``$RLB_REFIT_HOLD_FILE`` names an existing file, sleep until it is
    removed (or ``max_hold_s`` passes); returns the seconds held."""
    path = os.environ.get(HOLD_FILE_ENV)
    if not path:
        return 0.0
    t0 = time.monotonic()
    while os.path.exists(path) and time.monotonic() - t0 < max_hold_s:
        time.sleep(poll_s)
    return time.monotonic() - t0
