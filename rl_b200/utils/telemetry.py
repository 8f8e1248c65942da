"""Lightweight telemetry: nested spans with attributes, goodput accounting and a
JSONL exporter.

Reference: ``nemo_rl/telemetry`` (OpenTelemetry spans ``startup_span`` /
``setup_span`` / ``checkpoint_finalize_span``, goodput buckets,
``docs/observability``).  OpenTelemetry is not available here, so spans are
recorded in-process (start, end, parent, attributes) and written as JSON lines;
``goodput`` splits wall time into productive buckets (generation, log-prob,
training) and overhead (weight sync, checkpointing, data, idle).
"""

from __future__ import annotations

import contextlib
import json
import os
import threading
import time
from typing import Optional

__all__ = ["Telemetry", "PRODUCTIVE"]

PRODUCTIVE = ("generation", "policy_and_reference_logprobs", "policy_training")


class Telemetry:
    def __init__(self, path: Optional[str] = None, rank: int = 0):
        self.path = path
        self.rank = rank
        self.spans: list[dict] = []
        self._local = threading.local()
        self._t0 = time.time()

    @contextlib.contextmanager
    def span(self, name: str, **attrs):
        stack = getattr(self._local, "stack", None)
        if stack is None:
            stack = self._local.stack = []
        rec = {"name": name, "start": time.time(), "parent": stack[-1]["name"] if stack else None,
               "rank": self.rank, "attrs": attrs}
        stack.append(rec)
        try:
            yield rec
        finally:
            stack.pop()
            rec["end"] = time.time()
            rec["duration_s"] = rec["end"] - rec["start"]
            self.spans.append(rec)

    def goodput(self, timing: dict, step_time_s: float) -> dict:
        """``timing``: seconds per stage of one step (the GRPO timer's metrics)."""
        prod = sum(float(timing.get(k, 0.0)) for k in PRODUCTIVE)
        other = {k: float(v) for k, v in timing.items() if k not in PRODUCTIVE and k != "total_step_time"}
        idle = max(0.0, step_time_s - prod - sum(other.values()))
        out = {"goodput/productive_s": prod, "goodput/overhead_s": sum(other.values()), "goodput/idle_s": idle,
               "goodput/fraction": prod / step_time_s if step_time_s > 0 else 0.0}
        for k, v in other.items():
            out[f"goodput/overhead/{k}"] = v
        return out

    def flush(self) -> int:
        if not self.path or not self.spans:
            n = len(self.spans)
            self.spans.clear()
            return n
        os.makedirs(os.path.dirname(self.path) or ".", exist_ok=True)
        with open(self.path, "a") as f:
            for r in self.spans:
                f.write(json.dumps(r, default=str) + "\n")
        n = len(self.spans)
        self.spans.clear()
        return n
