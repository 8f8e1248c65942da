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


def _case_sparse(rank: int, port: int):
    from rl_b200.distributed.stateless_group import StatelessProcessGroup
    from rl_b200.weight_sync.broadcast import SparseDeltaBroadcastSynchronizer

    g = StatelessProcessGroup("127.0.0.1", port, rank, 3, backend="gloo", name="refit", timeout_s=30)
    n = 20000
    gen = torch.Generator().manual_seed(0)
    w = torch.randn(n, generator=gen).to(torch.bfloat16)
    flat = w.clone() if rank == 0 else torch.zeros(n, dtype=torch.bfloat16)
    ws = SparseDeltaBroadcastSynchronizer(flat, g, src=0, bucket_bytes=4096, timeout_s=20)
    out = {"full": ws.sync()}
    ok = [torch.equal(flat, w)]
    # a small update: most bf16 weights keep their bits, a few change
    upd = w.float() * (1 + 1e-4 * torch.randn(n, generator=gen))
    upd[::97] += 0.05  # some clearly changed entries
    upd[4096:6144] += 1.0  # one densely changed stretch (sent as whole buckets)
    upd = upd.to(torch.bfloat16)
    if rank == 0:
        flat.copy_(upd)
    out["delta"] = ws.sync()
    out["stats"] = ws.last_stats
    ok.append(torch.equal(flat, upd))
    out["no_change"] = ws.sync()
    ok.append(torch.equal(flat, upd))
    g.destroy()
    out["ok"] = all(ok)
    return out


def test_sparse_delta_refit_sends_only_changed_weights():
    """After one full refit, refits carry only the changed bf16 weights (positions
    + values, or whole buckets where most changed); every consumer ends with the
    producer's exact bits."""
    port = free_port()
    outs = spawn_ranks(_case_sparse, 3, port, timeout_s=120)
    assert all(o["ok"] for o in outs)
    o = outs[0]
    full = o["full"]["bytes"]
    assert full == 20000 * 2
    assert 0 < o["delta"]["bytes"] < 0.6 * full, o
    assert 0 < o["stats"]["changed_fraction"] < 0.5
    assert o["no_change"]["bytes"] <= 16 * (20000 * 2 // 4096 + 1)  # headers only
