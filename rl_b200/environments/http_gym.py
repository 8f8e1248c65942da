"""HTTP environment bridge (NeMo-Gym style) and an OpenAI-style completion server
over the in-house rollout engine.

``HttpGymEnvironment`` sends every sample of a ``step`` to an external
environment service as one JSON ``POST`` to ``{base_url}/run`` (concurrently,
``max_concurrency`` in flight):

    request  {"messages": [{"role", "content", "token_ids"}, ...],
              "metadata": <sample metadata>, "task": <task name>}
    response {"reward": float, "done": bool,
              "observation": {"role", "content"} | null, "metadata": <new metadata>,
              "invalid_tool_call": bool, "malformed_thinking": bool}

The two optional flags mark the sample's last assistant message
(``is_invalid_tool_call`` / ``has_malformed_thinking``) for GRPO's
message-level advantage penalties.

Failed calls are retried (``retries``) and then scored ``failure_reward`` with
the episode ended, so one bad row never stalls the batch.

``serve_policy`` exposes a rollout engine as ``POST /v1/completions`` taking
``prompt_token_ids`` (list of token-id lists) and returning per-choice
``token_ids`` and ``logprobs``, so agents inside the environment service can
call the policy being trained (token ids in and out; no tokenizer needed on
this side).

Reference: the NeMo-Gym integration (``nemo_rl/environments/nemo_gym.py:1122``
``NemoGym``, its ``/run`` calls ``:580`` and ``run_rollouts`` ``:1706``), whose
agents call the policy through an OpenAI-compatible model server.
"""

from __future__ import annotations

import json
import threading
import urllib.error
import urllib.request
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Optional

import torch

from rl_b200.environments.interfaces import EnvironmentInterface, EnvironmentReturn

__all__ = ["HttpGymEnvironment", "serve_policy"]


def _to_json(m: dict) -> dict:
    out = {"role": m.get("role"), "content": m.get("content", "")}
    if isinstance(m.get("token_ids"), torch.Tensor):
        out["token_ids"] = m["token_ids"].tolist()
    return out


class HttpGymEnvironment(EnvironmentInterface):
    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        self.base_url = str(cfg["base_url"]).rstrip("/")
        self.timeout = float(cfg.get("timeout_s", 60.0))
        self.retries = int(cfg.get("retries", 2))
        self.failure_reward = float(cfg.get("failure_reward", 0.0))
        self.task = cfg.get("task")
        self.pool = ThreadPoolExecutor(max_workers=int(cfg.get("max_concurrency", 64)))
        self.failures = 0

    def _post(self, payload: dict, carrier: Optional[dict] = None) -> Optional[dict]:
        body = json.dumps(payload).encode()
        # W3C trace context: the service's spans join the caller's trace
        headers = {"Content-Type": "application/json", **(carrier or {})}
        for _ in range(self.retries + 1):
            try:
                req = urllib.request.Request(self.base_url + "/run", data=body, headers=headers, method="POST")
                with urllib.request.urlopen(req, timeout=self.timeout) as r:
                    return json.loads(r.read().decode())
            except (urllib.error.URLError, TimeoutError, ValueError, OSError):
                continue
        return None

    def step(self, message_log_batch: list[list[dict]], metadata: list[Any]) -> EnvironmentReturn:
        payloads = [{"messages": [_to_json(m) for m in log], "metadata": md, "task": self.task}
                    for log, md in zip(message_log_batch, metadata)]
        from rl_b200.utils.telemetry import current_trace_carrier

        carrier = current_trace_carrier()  # captured here: the pool threads have their own context
        results = list(self.pool.map(lambda p: self._post(p, carrier), payloads))
        obs, meta, rewards, done = [], [], [], []
        for res, md, log in zip(results, metadata, message_log_batch):
            if res is None:
                self.failures += 1
                obs.append({})
                meta.append(md)
                rewards.append(self.failure_reward)
                done.append(True)
                continue
            obs.append(res.get("observation") or {})
            meta.append(res.get("metadata", md))
            last = next((m for m in reversed(log) if m.get("role") == "assistant"), None)
            if last is not None:
                if res.get("invalid_tool_call"):
                    last["is_invalid_tool_call"] = True
                if res.get("malformed_thinking"):
                    last["has_malformed_thinking"] = True
            rewards.append(float(res.get("reward", 0.0)))
            done.append(bool(res.get("done", True)))
        return EnvironmentReturn(obs, meta, [None] * len(obs), torch.tensor(rewards, dtype=torch.float32),
                                 torch.tensor(done, dtype=torch.bool))

    def global_post_process_and_metrics(self, batch):
        return batch, {"gym_failed_calls": float(self.failures)}

    def shutdown(self) -> None:
        self.pool.shutdown(wait=False)


def serve_policy(policy, host: str = "127.0.0.1", port: int = 0):
    """Serve ``policy.generate`` over HTTP (``POST /v1/completions``) on a
    background thread; returns ``(server, base_url)`` (``server.shutdown()`` stops it).
    Requests are executed one at a time on the caller's rollout engine."""
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    lock = threading.Lock()

    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *a):  # quiet
            pass

        def do_POST(self):  # noqa: N802 - http.server naming
            if self.path.rstrip("/") != "/v1/completions":
                self.send_error(404)
                return
            req = json.loads(self.rfile.read(int(self.headers.get("Content-Length", 0))).decode())
            prompts = req["prompt_token_ids"]
            if prompts and isinstance(prompts[0], int):
                prompts = [prompts]
            S = max(len(p) for p in prompts)
            ids = torch.zeros(len(prompts), S, dtype=torch.long)
            for i, p in enumerate(prompts):
                ids[i, :len(p)] = torch.tensor(p)
            data = BatchedDataDict({"input_ids": ids, "input_lengths": torch.tensor([len(p) for p in prompts])})
            with lock:
                out = policy.generate(data, greedy=float(req.get("temperature", 1.0)) == 0.0)
            choices = []
            for i, p in enumerate(prompts):
                n = int(out["generation_lengths"][i])
                L = len(p)
                choices.append({"index": i, "token_ids": out["output_ids"][i, L:L + n].tolist(),
                                "logprobs": out["logprobs"][i, L:L + n].tolist(),
                                "finish_reason": "length" if bool(out["truncated"][i]) else "stop"})
            body = json.dumps({"object": "text_completion", "choices": choices}).encode()
            self.send_response(200)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

    server = ThreadingHTTPServer((host, port), Handler)
    threading.Thread(target=server.serve_forever, daemon=True).start()
    return server, f"http://{host}:{server.server_address[1]}"
