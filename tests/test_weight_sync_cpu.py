"""Refit transports on CPU gloo ranks: bucketed broadcast over a stateless
(cross-world) group, and the watchdog aborting a refit held by host-side fault
injection (no GPU is involved, nothing hangs a device)."""

import os
import threading
import time

import torch

from rl_b200.distributed.launch import free_port, spawn_ranks


def _case_broadcast(rank: int, port: int):
    from rl_b200.distributed.stateless_group import StatelessProcessGroup
    from rl_b200.weight_sync.broadcast import PackedBroadcastSynchronizer

    g = StatelessProcessGroup("127.0.0.1", port, rank, 2, backend="gloo", name="refit", timeout_s=30)
    flat = torch.arange(10007, dtype=torch.float32) if rank == 0 else torch.zeros(10007)
    ws = PackedBroadcastSynchronizer(flat, g, src=0, bucket_bytes=4096, timeout_s=20)
    st = ws.sync()
    ok = torch.equal(flat, torch.arange(10007, dtype=torch.float32))
    g.destroy()
    return {"ok": ok, "bytes": st["bytes"], "aborted": ws.aborted}


def test_stateless_group_bucketed_broadcast():
    port = free_port()
    outs = spawn_ranks(_case_broadcast, 2, port, timeout_s=120)
    assert all(o["ok"] for o in outs) and not any(o["aborted"] for o in outs)
    assert outs[0]["bytes"] == 10007 * 4


def _case_watchdog(rank: int, port: int, hold_path: str):
    from rl_b200.distributed.stateless_group import GroupAborted, StatelessProcessGroup
    from rl_b200.weight_sync.broadcast import PackedBroadcastSynchronizer

    g = StatelessProcessGroup("127.0.0.1", port, rank, 2, backend="gloo", name="refit", timeout_s=30)
    flat = torch.ones(1000) if rank == 0 else torch.zeros(1000)
    if rank == 1:
        # this rank's refit is held (host-side) longer than the producer's deadline
        open(hold_path, "w").close()
        os.environ["RLB_REFIT_HOLD_FILE"] = hold_path
        threading.Timer(3.0, lambda: os.path.exists(hold_path) and os.remove(hold_path)).start()
    ws = PackedBroadcastSynchronizer(flat, g, src=0, timeout_s=1.0)
    t0 = time.monotonic()
    try:
        ws.sync()
        raised = False
    except GroupAborted:
        raised = True
    return {"raised": raised, "aborted": g.aborted, "elapsed": time.monotonic() - t0}


def test_refit_watchdog_aborts_held_refit(tmp_path):
    port = free_port()
    outs = spawn_ranks(_case_watchdog, 2, port, str(tmp_path / "hold"), timeout_s=120)
    # the producer gave up after its 1 s deadline instead of waiting for the held peer
    assert outs[0]["raised"] and outs[0]["aborted"] and outs[0]["elapsed"] < 2.9
    # the held rank, once released, finishes (data the producer had already sent)
    # or fails on its own deadline - it never waits for good
    assert outs[1]["elapsed"] < 10.0


def test_watchdog_context_and_hold(tmp_path, monkeypatch):
    from rl_b200.weight_sync.watchdog import RefitAbortWatchdog, hold_refit_for_fault_injection

    hits = []
    with RefitAbortWatchdog(0.2, lambda: hits.append(1)) as wd:
        time.sleep(0.5)
    assert wd.fired and hits == [1]
    with RefitAbortWatchdog(5.0, lambda: hits.append(2)) as wd:
        pass
    assert not wd.fired and hits == [1]
    p = tmp_path / "h"
    p.write_text("")
    monkeypatch.setenv("RLB_REFIT_HOLD_FILE", str(p))
    threading.Timer(0.3, p.unlink).start()
    held = hold_refit_for_fault_injection()
    assert 0.2 < held < 3.0
