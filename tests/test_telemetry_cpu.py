"""Tracing: W3C trace-context carriers across threads and HTTP, decorated
receivers, OTLP/JSON export to a file and to an HTTP collector, and the GRPO
loop's step traces (CPU)."""

from __future__ import annotations

import json
import os
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

from rl_b200.utils.telemetry import (Telemetry, accepts_trace_context, current_trace_carrier,
                                     dispatch_with_trace_context, parse_traceparent, read_otlp_spans,
                                     remote_trace_context)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_traceparent_parsing():
    tp = "00-" + "ab" * 16 + "-" + "cd" * 8 + "-01"
    assert parse_traceparent(tp) == ("ab" * 16, "cd" * 8)
    assert parse_traceparent("garbage") is None
    assert parse_traceparent("00-" + "0" * 32 + "-" + "cd" * 8 + "-01") is None


def test_carrier_links_spans_across_a_thread_and_a_decorated_call():
    t = Telemetry()
    out = {}

    @accepts_trace_context
    def worker_task(x):
        with t.span("remote_work"):
            out["x"] = x

    with t.span("parent") as parent:
        carrier = current_trace_carrier()
        th = threading.Thread(target=lambda: _in_thread(t, carrier))
        th.start()
        th.join()
        dispatch_with_trace_context(worker_task, 7)
    with t.span("unrelated"):
        pass
    by = {s.name: s for s in t.spans}
    assert by["child_in_thread"].parent_span_id == parent.span_id
    assert by["child_in_thread"].trace_id == parent.trace_id
    assert by["remote_work"].parent_span_id == parent.span_id and out["x"] == 7
    assert by["unrelated"].trace_id != parent.trace_id and by["unrelated"].parent_span_id is None


def _in_thread(t, carrier):
    assert current_trace_carrier() == {}  # a new thread starts with no span
    with remote_trace_context(carrier):
        with t.span("child_in_thread"):
            pass


class _Collector(BaseHTTPRequestHandler):
    bodies: list = []
    headers_seen: list = []

    def do_POST(self):  # noqa: N802
        n = int(self.headers["Content-Length"])
        body = json.loads(self.rfile.read(n))
        type(self).bodies.append((self.path, body))
        type(self).headers_seen.append({k.lower(): v for k, v in self.headers.items()})
        reply = json.dumps({"reward": 1.0, "done": True}).encode() if self.path == "/run" else b"{}"
        self.send_response(200)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(reply)))
        self.end_headers()
        self.wfile.write(reply)

    def log_message(self, *a):
        pass


def test_otlp_http_export_and_http_environment_propagation(tmp_path):
    import torch

    from rl_b200.environments.http_gym import HttpGymEnvironment

    srv = HTTPServer(("127.0.0.1", 0), _Collector)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{srv.server_address[1]}"
    try:
        t = Telemetry(str(tmp_path / "t.jsonl"), otlp_endpoint=url + "/v1/traces")
        env = HttpGymEnvironment({"base_url": url, "timeout_s": 5})
        with t.span("rollout") as sp:
            env.step([[{"role": "assistant", "content": "hi", "token_ids": torch.tensor([1, 2])}]], [{}])
        assert t.flush() == 1
        runs = [h for (path, _), h in zip(_Collector.bodies, _Collector.headers_seen) if path == "/run"]
        assert runs and parse_traceparent(runs[0]["traceparent"]) == (sp.trace_id, sp.span_id)
        exported = [b for path, b in _Collector.bodies if path == "/v1/traces"]
        assert exported and exported[0]["resourceSpans"][0]["scopeSpans"][0]["spans"][0]["name"] == "rollout"
        assert read_otlp_spans(str(tmp_path / "t.jsonl"))[0]["spanId"] == sp.span_id
    finally:
        srv.shutdown()


def test_grpo_writes_step_traces(tmp_path):
    from examples.run_grpo import main

    path = str(tmp_path / "trace.jsonl")
    main(["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
          "logger.log_dir=" + str(tmp_path / "logs"), "logger.stdout=false", f"++telemetry.path={path}"])
    spans = read_otlp_spans(path)
    steps = [s for s in spans if s["name"] == "step"]
    assert len(steps) == 2
    gen = [s for s in spans if s["name"] == "generation"]
    assert {g["parentSpanId"] for g in gen} == {s["spanId"] for s in steps}
