"""HTTP router in front of the generation fleet.

Reference: ``nemo_rl/models/generation/generation_router.py:65``
(``GenerationRouterImpl``: one stable URL handed to the environment service,
``set_serving_backends`` from the fleet health, per-request least-outstanding
backend choice, requests forwarded (not redirected) so a backend that dies
mid-request is failed over inside the router, ``drain_backend_outcomes`` of
per-backend successes / failures for the health state machine, ``metrics``).

Here the router is a threaded ``http.server`` on a port fixed at construction
(so it can be rebuilt on the same URL); each request body is forwarded to the
serving backend with the fewest requests in flight, and on a connection error
or a 5xx reply to the next one (each backend tried once), with the outcome
recorded.  ``attach_fleet`` wires it to ``GenerationFleetHealth``: outcomes
update the shards' states and the serving set follows ``serving_shards``.
"""

from __future__ import annotations

import threading
import urllib.error
import urllib.request
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Optional

__all__ = ["GenerationRouter"]

_SKIP_REQUEST = frozenset({"host", "content-length", "connection"})
_SKIP_RESPONSE = frozenset({"content-length", "transfer-encoding", "connection", "server", "date"})


class GenerationRouter:
    def __init__(self, host: str = "127.0.0.1", port: int = 0, backend_timeout_s: float = 600.0,
                 no_healthy_backend_status: int = 409):
        self.backend_timeout_s = float(backend_timeout_s)
        self.no_backend_status = int(no_healthy_backend_status)
        self._lock = threading.Lock()
        self._backends: list[str] = []
        self._inflight: dict[str, int] = {}
        self._outcomes: dict[str, list[int]] = {}   # backend -> [successes, failures] since the last drain
        self._stats = {"requests": 0, "failovers": 0, "no_backend": 0, "errors": 0}
        self._fleet = None
        self._fleet_urls: list[str] = []
        router = self

        class Handler(BaseHTTPRequestHandler):
            protocol_version = "HTTP/1.1"

            def log_message(self, *a):  # quiet
                pass

            def _handle(self, method: str):
                n = int(self.headers.get("Content-Length", 0) or 0)
                body = self.rfile.read(n) if n else None
                headers = {k: v for k, v in self.headers.items() if k.lower() not in _SKIP_REQUEST}
                status, rheaders, payload = router._route(method, self.path, headers, body)
                self.send_response(status)
                for k, v in rheaders:
                    if k.lower() not in _SKIP_RESPONSE:
                        self.send_header(k, v)
                self.send_header("Content-Length", str(len(payload)))
                self.end_headers()
                self.wfile.write(payload)

            def do_POST(self):  # noqa: N802 - http.server naming
                self._handle("POST")

            def do_GET(self):  # noqa: N802
                self._handle("GET")

        self._server = ThreadingHTTPServer((host, port), Handler)
        self._server.daemon_threads = True
        self._thread: Optional[threading.Thread] = None

    # ------------------------------------------------------------ lifecycle
    @property
    def base_url(self) -> str:
        h, p = self._server.server_address[:2]
        return f"http://{h}:{p}"

    def serve_in_background(self) -> "GenerationRouter":
        if self._thread is None:
            self._thread = threading.Thread(target=self._server.serve_forever, name="generation-router", daemon=True)
            self._thread.start()
        return self

    def shutdown(self) -> None:
        self._server.shutdown()
        self._server.server_close()

    # -------------------------------------------------------------- backends
    def set_serving_backends(self, urls: list[str]) -> None:
        """Replace the serving set (in-flight counts of kept backends survive)."""
        with self._lock:
            self._backends = [u.rstrip("/") for u in urls]
            self._inflight = {u: self._inflight.get(u, 0) for u in self._backends}

    def attach_fleet(self, fleet, urls: list[str]) -> None:
        """Route over ``fleet``'s serving shards (shard ``i`` at ``urls[i]``) and
        report every forwarded request's outcome to it."""
        self._fleet, self._fleet_urls = fleet, [u.rstrip("/") for u in urls]
        self.refresh_from_fleet()

    def refresh_from_fleet(self) -> None:
        if self._fleet is not None:
            self.set_serving_backends([self._fleet_urls[i] for i in self._fleet.serving_shards()])

    def drain_backend_outcomes(self) -> dict[str, tuple[int, int]]:
        """Per-backend (successes, failures) since the previous drain."""
        with self._lock:
            out = {u: (s, f) for u, (s, f) in self._outcomes.items()}
            self._outcomes = {}
        return out

    def metrics(self) -> dict[str, float]:
        with self._lock:
            m = {f"generation_router/{k}": float(v) for k, v in self._stats.items()}
            m["generation_router/serving_backends"] = float(len(self._backends))
            m["generation_router/inflight"] = float(sum(self._inflight.values()))
        return m

    # --------------------------------------------------------------- routing
    def _candidates(self) -> list[str]:
        with self._lock:  # least outstanding first (ties: list order)
            return sorted(self._backends, key=lambda u: self._inflight.get(u, 0))

    def _record(self, url: str, ok: bool) -> None:
        with self._lock:
            s, f = self._outcomes.get(url, [0, 0])
            self._outcomes[url] = [s + int(ok), f + int(not ok)]
        if self._fleet is not None and url in self._fleet_urls:
            i = self._fleet_urls.index(url)
            if ok:
                self._fleet.report_success(i)
            else:
                self._fleet.report_failure(i, "request failed through the generation router")
            self.refresh_from_fleet()

    def _route(self, method: str, path: str, headers: dict, body: Optional[bytes]):
        with self._lock:
            self._stats["requests"] += 1
        tried = 0
        for url in self._candidates():
            with self._lock:
                if url not in self._inflight:
                    continue  # dropped from the serving set meanwhile
                self._inflight[url] += 1
            tried += 1
            try:
                req = urllib.request.Request(url + path, data=body, headers=headers, method=method)
                with urllib.request.urlopen(req, timeout=self.backend_timeout_s) as r:
                    payload = r.read()
                    status, rheaders = r.status, list(r.headers.items())
                self._record(url, True)
                return status, rheaders, payload
            except urllib.error.HTTPError as e:
                if e.code < 500:  # the request itself was refused: no failover, pass it through
                    self._record(url, True)
                    return e.code, list(e.headers.items()), e.read()
                self._record(url, False)
            except (urllib.error.URLError, OSError):
                self._record(url, False)
            finally:
                with self._lock:
                    if url in self._inflight:
                        self._inflight[url] -= 1
            with self._lock:
                self._stats["failovers"] += 1
        with self._lock:
            self._stats["no_backend" if tried == 0 else "errors"] += 1
        msg = b'{"error": "no healthy generation backend"}'
        return (self.no_backend_status if tried == 0 else 502), [("Content-Type", "application/json")], msg
