"""HTTP environment bridge against a local environment service, and the policy
completion server an agent inside the service would call."""

import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import torch


def _gym_server(policy_url=None):
    """A toy environment service: reward = fraction of even token ids in the
    assistant turns; optionally asks the policy for one more completion."""
    calls = {"n": 0}

    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_POST(self):
            req = json.loads(self.rfile.read(int(self.headers["Content-Length"])).decode())
            calls["n"] += 1
            toks = [t for m in req["messages"] if m["role"] == "assistant" for t in m.get("token_ids", [])]
            extra = 0
            if policy_url is not None:
                import urllib.request

                body = json.dumps({"prompt_token_ids": [toks[:4] or [1]], "temperature": 0.0}).encode()
                r = urllib.request.urlopen(urllib.request.Request(policy_url + "/v1/completions", data=body,
                                                                  headers={"Content-Type": "application/json"}))
                extra = len(json.loads(r.read())["choices"][0]["token_ids"])
            reward = sum(t % 2 == 0 for t in toks) / max(1, len(toks))
            out = json.dumps({"reward": reward, "done": True, "metadata": {"extra": extra}}).encode()
            self.send_response(200)
            self.send_header("Content-Length", str(len(out)))
            self.end_headers()
            self.wfile.write(out)

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, f"http://127.0.0.1:{srv.server_address[1]}", calls


def test_http_gym_environment_and_policy_server():
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.environments.http_gym import serve_policy
    from rl_b200.environments.registry import make_environment
    from rl_b200.experience.rollouts import run_multi_turn_rollout
    from tests.test_core_cpu import _tiny_policy

    w = _tiny_policy(seed=5)
    psrv, purl = serve_policy(w)
    gsrv, gurl, calls = _gym_server(purl)
    try:
        env = make_environment("nemo_gym", {"base_url": gurl, "max_concurrency": 4})
        g = torch.Generator().manual_seed(0)
        logs = [[{"role": "user", "content": "", "token_ids": torch.randint(0, 512, (6,), generator=g)}]
                for _ in range(4)]
        batch = BatchedDataDict({"message_log": logs, "task_name": ["gym"] * 4, "extra_env_info": [None] * 4,
                                 "loss_multiplier": torch.ones(4)})
        rollout, _ = run_multi_turn_rollout(w, batch, None, {"gym": env}, 48)
        assert calls["n"] == 4
        for i, log in enumerate(rollout["message_log"]):
            toks = log[-1]["token_ids"].tolist()
            assert abs(float(rollout["total_reward"][i]) - sum(t % 2 == 0 for t in toks) / len(toks)) < 1e-6
            assert rollout["extra_env_info"][i]["extra"] >= 1  # the service called the policy server
        # an unreachable service scores the failure reward instead of raising
        bad = make_environment("http_gym", {"base_url": "http://127.0.0.1:9", "retries": 0, "timeout_s": 2,
                                            "failure_reward": -1.0})
        ret = bad.step(logs[:2], [None, None])
        assert ret.rewards.tolist() == [-1.0, -1.0] and bool(ret.terminateds.all())
    finally:
        gsrv.shutdown()
        psrv.shutdown()
