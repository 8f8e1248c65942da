"""Tracing and goodput telemetry with W3C trace-context propagation and an
OTLP/JSON exporter.

Reference: ``nemo_rl/telemetry`` (OpenTelemetry spans through nemo-lens:
``managed_span`` / ``trace_fn``, the ``rl.bucket`` efficiency tag
(productive | overhead | idle | wasted), carrier propagation across process
boundaries ``current_trace_carrier`` / ``remote_trace_context`` /
``accepts_trace_context`` / ``dispatch_with_trace_context``,
``instrumentation.py:411-660``, and goodput accounting).  OpenTelemetry is not
installed in this image, so the data model is implemented here directly:

* spans carry a 128-bit trace id, a 64-bit span id and the parent span id; the
  current span lives in a ``contextvars`` variable, so nesting follows the
  call stack within a thread or asyncio task;
* a carrier is the W3C ``traceparent`` header (``00-<trace>-<span>-01``): it is
  what crosses a thread, a process or an HTTP request (the HTTP environment
  bridge sends it), and ``remote_trace_context(carrier)`` makes spans opened on
  the other side children of the sender's span;
* finished spans export as OTLP/JSON ``resourceSpans`` (the encoding an
  OpenTelemetry collector's file or OTLP/HTTP receiver accepts): appended to a
  file, and POSTed to ``otlp_endpoint`` (``.../v1/traces``) when one is set.
"""

from __future__ import annotations

import contextlib
import contextvars
import functools
import json
import os
import re
import secrets
import threading
import time
import urllib.request
from dataclasses import dataclass, field
from typing import Any, Callable, Iterator, Mapping, Optional

__all__ = ["Telemetry", "PRODUCTIVE", "Span", "RL_BUCKET_ATTR", "bucket_for_stage", "current_span",
           "current_trace_carrier", "remote_trace_context", "accepts_trace_context", "dispatch_with_trace_context",
           "TRACE_CARRIER_KWARG", "parse_traceparent", "read_otlp_spans"]

PRODUCTIVE = ("generation", "policy_and_reference_logprobs", "policy_training")
RL_BUCKET_ATTR = "rl.bucket"
TRACE_CARRIER_KWARG = "_trace_carrier"
_BUCKETS = {"generation": "productive", "policy_and_reference_logprobs": "productive",
            "policy_training": "productive", "weight_sync": "overhead", "checkpointing": "overhead",
            "data_processing": "overhead", "validation": "overhead", "exposed_generation": "idle",
            "discarded_generation": "wasted"}
_TRACEPARENT = re.compile(r"^00-([0-9a-f]{32})-([0-9a-f]{16})-([0-9a-f]{2})$")


def bucket_for_stage(stage: str) -> Optional[str]:
    """Efficiency bucket of a timed stage name (None: an umbrella, not tagged)."""
    return _BUCKETS.get(stage)


@dataclass
class Span:
    name: str
    trace_id: str
    span_id: str
    parent_span_id: Optional[str]
    start_ns: int
    end_ns: Optional[int] = None
    attributes: dict = field(default_factory=dict)
    status: str = "ok"

    def set_attribute(self, key: str, value: Any) -> None:
        self.attributes[key] = value

    @property
    def traceparent(self) -> str:
        return f"00-{self.trace_id}-{self.span_id}-01"


_CURRENT: contextvars.ContextVar[Optional[Span]] = contextvars.ContextVar("rlb_current_span", default=None)
# remote parent (trace id, span id) attached by remote_trace_context, used when no local span is open
_REMOTE: contextvars.ContextVar[Optional[tuple[str, str]]] = contextvars.ContextVar("rlb_remote_parent",
                                                                                   default=None)


def parse_traceparent(value: str) -> Optional[tuple[str, str]]:
    """(trace id, parent span id) of a W3C traceparent header, or None if malformed."""
    m = _TRACEPARENT.match((value or "").strip().lower())
    if not m or m.group(1) == "0" * 32 or m.group(2) == "0" * 16:
        return None
    return m.group(1), m.group(2)


def current_span() -> Optional[Span]:
    return _CURRENT.get()


def current_trace_carrier() -> dict[str, str]:
    """``{"traceparent": ...}`` of the span open in this context ({} when none)."""
    sp = _CURRENT.get()
    if sp is not None:
        return {"traceparent": sp.traceparent}
    rp = _REMOTE.get()
    return {"traceparent": f"00-{rp[0]}-{rp[1]}-01"} if rp else {}


@contextlib.contextmanager
def remote_trace_context(carrier: Optional[Mapping[str, str]]) -> Iterator[None]:
    """Spans opened inside become children of the carrier's span (a span of
    another thread, process or service); a missing or malformed carrier starts
    nothing new (spans then root their own trace)."""
    parent = parse_traceparent((carrier or {}).get("traceparent", "")) if carrier else None
    t1 = _REMOTE.set(parent)
    t2 = _CURRENT.set(None)
    try:
        yield
    finally:
        _CURRENT.reset(t2)
        _REMOTE.reset(t1)


def accepts_trace_context(fn: Callable) -> Callable:
    """Decorate a function that may be called with ``_trace_carrier=...``: the
    keyword is removed and the call runs under that remote parent."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        carrier = kwargs.pop(TRACE_CARRIER_KWARG, None)
        if carrier is None:
            return fn(*args, **kwargs)
        with remote_trace_context(carrier):
            return fn(*args, **kwargs)

    wrapper.__rlb_accepts_trace_context__ = True
    return wrapper


def dispatch_with_trace_context(fn: Callable, /, *args, **kwargs):
    """Call ``fn`` (a function run on another thread / worker) with the caller's
    carrier when it accepts one; otherwise call it unchanged."""
    carrier = current_trace_carrier()
    if carrier and getattr(fn, "__rlb_accepts_trace_context__", False):
        kwargs[TRACE_CARRIER_KWARG] = carrier
    return fn(*args, **kwargs)


def _otlp_value(v: Any) -> dict:
    if isinstance(v, bool):
        return {"boolValue": v}
    if isinstance(v, int):
        return {"intValue": str(v)}
    if isinstance(v, float):
        return {"doubleValue": v}
    return {"stringValue": str(v)}


class Telemetry:
    """Span recorder of one process.

    ``span(name, **attrs)`` opens a child of the current span (or of the remote
    parent attached by ``remote_trace_context``, or a new trace); a stage name
    with an efficiency bucket gets ``rl.bucket``.  ``flush()`` writes the
    finished spans (OTLP/JSON to ``path``; also POSTed to ``otlp_endpoint``) and
    returns how many.  ``goodput`` splits a step's wall time into productive
    stages, overhead stages and idle time."""

    def __init__(self, path: Optional[str] = None, rank: int = 0, service_name: str = "rl_b200",
                 otlp_endpoint: Optional[str] = None, resource: Optional[dict] = None):
        self.path = path
        self.rank = rank
        self.service_name = service_name
        self.otlp_endpoint = otlp_endpoint or os.environ.get("RLB_OTLP_ENDPOINT")
        self.resource = {"service.name": service_name, "rl.rank": rank, **(resource or {})}
        self.spans: list[Span] = []
        self._lock = threading.Lock()

    @contextlib.contextmanager
    def span(self, name: str, **attrs) -> Iterator[Span]:
        parent = _CURRENT.get()
        if parent is not None:
            trace_id, parent_id = parent.trace_id, parent.span_id
        else:
            rp = _REMOTE.get()
            trace_id, parent_id = (rp if rp else (secrets.token_hex(16), None))
        sp = Span(name, trace_id, secrets.token_hex(8), parent_id, time.time_ns(), attributes=dict(attrs))
        b = bucket_for_stage(name)
        if b is not None:
            sp.attributes.setdefault(RL_BUCKET_ATTR, b)
        token = _CURRENT.set(sp)
        try:
            yield sp
        except BaseException as e:
            sp.status = "error"
            sp.attributes["exception.type"] = type(e).__name__
            raise
        finally:
            _CURRENT.reset(token)
            sp.end_ns = time.time_ns()
            with self._lock:
                self.spans.append(sp)

    def record_stage_spans(self, timing: dict, parent: Optional[Span] = None) -> None:
        """Spans for a step's timed stages (seconds each, the loop timer's output),
        laid end to end under ``parent`` (default: the current span): a trace of a
        step that was timed with a plain timer."""
        parent = parent or _CURRENT.get()
        if parent is None:
            return
        t = parent.start_ns
        for stage, secs in timing.items():
            if stage == "total_step_time":
                continue
            d = int(float(secs) * 1e9)
            sp = Span(stage, parent.trace_id, secrets.token_hex(8), parent.span_id, t, t + d)
            b = bucket_for_stage(stage)
            if b is not None:
                sp.attributes[RL_BUCKET_ATTR] = b
            t += d
            with self._lock:
                self.spans.append(sp)

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

    def to_otlp(self, spans: list[Span]) -> dict:
        """OTLP/JSON ``ExportTraceServiceRequest`` body for ``spans``."""
        out = []
        for s in spans:
            d = {"traceId": s.trace_id, "spanId": s.span_id, "name": s.name, "kind": 1,
                 "startTimeUnixNano": str(s.start_ns), "endTimeUnixNano": str(s.end_ns or s.start_ns),
                 "attributes": [{"key": k, "value": _otlp_value(v)} for k, v in s.attributes.items()],
                 "status": {"code": 2 if s.status == "error" else 1}}
            if s.parent_span_id:
                d["parentSpanId"] = s.parent_span_id
            out.append(d)
        return {"resourceSpans": [{
            "resource": {"attributes": [{"key": k, "value": _otlp_value(v)} for k, v in self.resource.items()]},
            "scopeSpans": [{"scope": {"name": "rl_b200.telemetry"}, "spans": out}]}]}

    def flush(self) -> int:
        with self._lock:
            spans, self.spans = self.spans, []
        if not spans:
            return 0
        body = self.to_otlp(spans)
        if self.path:
            os.makedirs(os.path.dirname(self.path) or ".", exist_ok=True)
            with open(self.path, "a") as f:
                f.write(json.dumps(body) + "\n")
        if self.otlp_endpoint:
            req = urllib.request.Request(self.otlp_endpoint, data=json.dumps(body).encode(),
                                         headers={"Content-Type": "application/json"}, method="POST")
            try:
                with urllib.request.urlopen(req, timeout=10) as r:
                    r.read()
            except OSError:  # an unreachable collector must not stop training
                pass
        return len(spans)


def read_otlp_spans(path: str) -> list[dict]:
    """Flattened spans of an OTLP/JSON file written by ``Telemetry.flush``."""
    out = []
    with open(path) as f:
        for line in f:
            for rs in json.loads(line)["resourceSpans"]:
                for ss in rs["scopeSpans"]:
                    out.extend(ss["spans"])
    return out
