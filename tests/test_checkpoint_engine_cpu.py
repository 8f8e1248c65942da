"""Checkpoint-engine weight transfer between a policy process and a rollout
process with no shared process group (shared-memory slots + key-value store):
chunking of tensors larger than a bucket, two-slot flow control across many
buckets, two refits, and the synchronizer loading into a second model (CPU)."""

from __future__ import annotations

import multiprocessing as mp

import torch

from rl_b200.weight_sync.checkpoint_engine import (TensorMeta, create_checkpoint_engine, merge_weight_chunk_batches,
                                                   split_weight_chunks)


def test_split_and_merge_round_trip():
    ws = [("a", torch.arange(10, dtype=torch.float32)), ("b", torch.randn(3, 5)), ("c", torch.zeros(0))]
    chunks = list(split_weight_chunks(ws, 16))
    assert all(m.chunk_size <= 16 for m, _ in chunks)
    assert [m.name for m, _ in chunks].count("a") == 3  # 40 bytes in 16-byte chunks
    batches = [[c] for c in chunks]  # one chunk per received batch
    got = dict(kv for b in merge_weight_chunk_batches(batches) for kv in b)
    for name, w in ws:
        assert torch.equal(got[name], w)
    assert TensorMeta("x", torch.Size([2, 3]), torch.bfloat16, 0, 12, 0).nbytes == 12


def _tiny():
    from rl_b200.models.config import ModelConfig

    return ModelConfig(name="ce", vocab_size=96, hidden_size=32, num_layers=2, num_heads=2, num_kv_heads=1,
                       head_dim=16, ffn_hidden_size=64, rope_theta=10000.0, max_position_embeddings=64)


def _policy(q_meta, q_port, q_done):
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.weight_sync.checkpoint_engine import CheckpointEngineSynchronizer

    eng = create_checkpoint_engine("shm", bucket_size_bytes=4096,
                                   engine_kwargs={"is_master": True, "port": 0, "timeout_s": 60})
    meta = eng.prepare()
    eng.init_policy_process_group(worker_rank=0, train_world_size=1, rollout_world_size=1, metadata=[meta])
    q_meta.put(meta)
    q_port.put(eng.port)
    m = TransformerLM(_tiny(), device="cpu", dtype=torch.float32, seed=3)
    sync = CheckpointEngineSynchronizer(eng, m)
    sync.sync()
    with torch.no_grad():
        m.flat_param.mul_(2.0)  # second weight version
    sync.sync()
    q_done.get(timeout=60)  # the rollout side finished reading
    eng.close(unlink=True)


def _rollout(meta, port, q_out):
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.weight_sync.checkpoint_engine import CheckpointEngineSynchronizer

    eng = create_checkpoint_engine("shm", bucket_size_bytes=4096, engine_kwargs={"port": port, "timeout_s": 60})
    eng.init_rollout_process_group(rollout_rank=0, train_world_size=1, rollout_world_size=1, metadata=[meta])
    m = TransformerLM(_tiny(), device="cpu", dtype=torch.float32, seed=99)
    sync = CheckpointEngineSynchronizer(eng, m)
    ref = TransformerLM(_tiny(), device="cpu", dtype=torch.float32, seed=3)
    n1 = sync.receive_into(m)
    ok1 = torch.equal(m.flat_param, ref.flat_param)
    n2 = sync.receive_into(m)
    ok2 = torch.equal(m.flat_param, ref.flat_param * 2.0)
    q_out.put((n1, n2, ok1, ok2, eng.seq))
    eng.close()


def test_shared_memory_engine_two_processes():
    ctx = mp.get_context("spawn")
    q_meta, q_port, q_done, q_out = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    pp = ctx.Process(target=_policy, args=(q_meta, q_port, q_done))
    pp.start()
    meta = q_meta.get(timeout=120)
    port = q_port.get(timeout=60)
    rp = ctx.Process(target=_rollout, args=(meta, port, q_out))
    rp.start()
    n1, n2, ok1, ok2, buckets = q_out.get(timeout=180)
    q_done.put(True)
    rp.join(60)
    pp.join(60)
    assert ok1 and ok2 and n1 == n2 > 0
    assert buckets > 4  # the model crossed many 4 KiB buckets (two-slot flow control exercised)
    assert pp.exitcode == 0 and rp.exitcode == 0
