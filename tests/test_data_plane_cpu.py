"""Data plane: codec round trip, in-process plane with a blocking consumer
thread, Store-backed plane across two processes, and a GRPO run whose train
batches flow through the plane."""

import os
import socket
import threading

import torch

from rl_b200.data_plane import InProcessDataPlane, decode_batch, encode_batch
from rl_b200.distributed.batched_data_dict import BatchedDataDict

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_codec_and_in_process_plane():
    b = BatchedDataDict({"x": torch.randn(3, 5).to(torch.bfloat16), "i": torch.arange(7), "m": [{"a": 1}, None],
                         "f8": torch.randn(2, 16).to(torch.float8_e4m3fn)})
    for z in (False, True):
        d = decode_batch(encode_batch(b, z))
        assert torch.equal(d["x"], b["x"]) and torch.equal(d["i"], b["i"]) and d["m"] == b["m"]
        assert torch.equal(d["f8"].view(torch.uint8), b["f8"].view(torch.uint8))
    dp = InProcessDataPlane()
    got = {}
    t = threading.Thread(target=lambda: got.setdefault("v", dp.get("p", "k", timeout=10)))
    t.start()
    dp.put("p", "k", b)  # the consumer was already waiting
    t.join()
    assert torch.equal(got["v"]["i"], b["i"]) and dp.keys("p") == ["k"]
    dp.delete("p", "k")
    assert dp.keys("p") == []
    try:
        dp.get("p", "missing", timeout=0.1)
        raise AssertionError("expected a timeout")
    except TimeoutError:
        pass


def test_store_plane_two_processes():
    from rl_b200.distributed.launch import spawn_ranks
    from tests.dist_cases import case_data_plane

    for attempt in range(3):  # a port picked this way can be taken again before the store binds it
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
        s.close()
        try:
            outs = spawn_ranks(case_data_plane, 2, port)
            break
        except RuntimeError:
            if attempt == 2:
                raise
    assert all(o["ok"] for o in outs)
    assert outs[0]["stats"]["data_plane/puts"] == 1 and outs[0]["stats"]["data_plane/gets"] == 1


def test_grpo_through_data_plane():
    from examples.run_grpo import main

    state = main(["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  "logger.log_dir=/tmp/rlb_test_logs_dp", "logger.stdout=false", "grpo.max_num_steps=1",
                  "++data_plane.enabled=true", "++data_plane.backend=in_process"])
    assert state["current_step"] == 1
