"""Generation router (CPU): one stable URL over the serving backends,
least-outstanding choice, failover when a backend dies, 4xx passed through,
the no-backend status, and the fleet-health wiring that retires a failing shard."""

from __future__ import annotations

import json
import threading
import time
import urllib.error
import urllib.request
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest

from rl_b200.models.generation.fleet_health import FleetHealthPolicy, GenerationFleetHealth, ShardState
from rl_b200.models.generation.router import GenerationRouter


def _backend(name: str, delay: float = 0.0):
    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_POST(self):  # noqa: N802
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            if body.get("bad"):
                self.send_error(400, "bad request")
                return
            time.sleep(delay)
            out = json.dumps({"backend": name, "echo": body}).encode()
            self.send_response(200)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(out)))
            self.end_headers()
            self.wfile.write(out)

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, f"http://127.0.0.1:{srv.server_address[1]}"


def _post(url, payload):
    req = urllib.request.Request(url + "/v1/completions", data=json.dumps(payload).encode(),
                                 headers={"Content-Type": "application/json"}, method="POST")
    with urllib.request.urlopen(req, timeout=10) as r:
        return r.status, json.loads(r.read())


def test_router_balances_fails_over_and_reports():
    a, ua = _backend("a")
    b, ub = _backend("b")
    r = GenerationRouter().serve_in_background()
    try:
        with pytest.raises(urllib.error.HTTPError) as e:  # no backend yet
            _post(r.base_url, {"x": 1})
        assert e.value.code == 409
        r.set_serving_backends([ua, ub])
        seen = {_post(r.base_url, {"x": i})[1]["backend"] for i in range(6)}
        assert seen == {"a"}  # sequential calls: nothing outstanding, ties go to the first backend
        with pytest.raises(urllib.error.HTTPError) as e:  # a refused request is not failed over
            _post(r.base_url, {"bad": True})
        assert e.value.code == 400
        a.shutdown()
        a.server_close()
        st, out = _post(r.base_url, {"x": 99})
        assert st == 200 and out["backend"] == "b" and out["echo"] == {"x": 99}
        oc = r.drain_backend_outcomes()
        assert oc[ua][1] >= 1 and oc[ub][0] >= 1
        assert r.metrics()["generation_router/failovers"] >= 1
    finally:
        r.shutdown()
        b.shutdown()


def test_concurrent_requests_use_least_outstanding_backends():
    a, ua = _backend("a", delay=0.3)
    b, ub = _backend("b", delay=0.3)
    r = GenerationRouter().serve_in_background()
    r.set_serving_backends([ua, ub])
    got = []
    ts = [threading.Thread(target=lambda i=i: got.append(_post(r.base_url, {"i": i})[1]["backend"]))
          for i in range(4)]
    try:
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert sorted(got).count("a") == 2 and sorted(got).count("b") == 2
    finally:
        r.shutdown()
        a.shutdown()
        b.shutdown()


def test_router_follows_fleet_health():
    a, ua = _backend("a")
    b, ub = _backend("b")
    fleet = GenerationFleetHealth(2, FleetHealthPolicy(unhealthy_threshold=2))
    r = GenerationRouter().serve_in_background()
    r.attach_fleet(fleet, [ua, ub])
    try:
        a.shutdown()
        a.server_close()
        for i in range(3):
            assert _post(r.base_url, {"i": i})[1]["backend"] == "b"
        assert fleet.state_of(0) == ShardState.DEAD and fleet.serving_shards() == [1]
        assert r.metrics()["generation_router/serving_backends"] == 1.0
    finally:
        r.shutdown()
        b.shutdown()
