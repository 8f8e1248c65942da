"""Fused compute + collective paths against their NCCL baselines, timed on the
device (CUDA events, 3 warm-up and 10 timed calls, max over ranks), with the
NVLink roofline of each: the bytes that must cross one GPU's link in one
direction divided by the measured 770 GB/s peer-copy bandwidth.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \\
        --master-addr 127.0.0.1 --master-port 29541 -m rl_b200.bench_collectives

Paths (two ranks):

* EP dispatch + combine (``csrc/ep_comm.cu`` peer stores): T tokens per rank,
  top-k of E experts split over the ranks, rows of H bf16; baseline: NCCL
  all-to-all of the same rows there and back.
* DP reduce-scatter + AdamW + parameter all-gather (``csrc/dp_optim.cu``) over a
  flat fp32 gradient / bf16 parameter buffer; baseline: NCCL reduce-scatter,
  the same AdamW kernel on the shard, NCCL all-gather.
* TP decode all-reduce + residual add + RMSNorm (``csrc/decode_ar.cu``) of a
  ``[B, H]`` bf16 partial; baseline: NCCL all-reduce then the fused add + RMSNorm.
"""

from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy, GB/s per direction


def _timeit(fn, reps: int = 10, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bench_ep(T: int = 4096, H: int = 2048, E: int = 128, k: int = 8) -> dict:
    from rl_b200.parallel.ep_fused import EPExchange, ep_combine, ep_dispatch, make_plan

    n, me = dist.get_world_size(), dist.get_rank()
    g = torch.Generator(device="cuda").manual_seed(100 + me)
    h = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.rand(T, E, device="cuda", generator=g).argsort(-1)[:, :k]  # k distinct experts per token
    plan = make_plan(ids, n, me, E // n, dist.group.WORLD)
    ex = (EPExchange(dist.group.WORLD, plan.R_max + 128, H), EPExchange(dist.group.WORLD, plan.TK_max + 128, H))

    def fused():
        xr = ep_dispatch(h, plan, ex[0], ex[1])
        ep_combine(xr, plan, ex[0], ex[1])

    # NCCL baseline: rows grouped by destination rank, all-to-all there and back
    dst = (ids.reshape(-1) // (E // n))
    order = torch.argsort(dst, stable=True)
    send = h[order // k]
    splits = torch.bincount(dst, minlength=n)
    all_s = torch.empty(n * n, dtype=splits.dtype, device="cuda")
    dist.all_gather_into_tensor(all_s, splits)
    send_l = splits.tolist()
    recv_l = all_s.view(n, n)[:, me].tolist()
    recv = torch.empty(sum(recv_l), H, dtype=torch.bfloat16, device="cuda")
    back = torch.empty_like(send)

    def nccl():
        dist.all_to_all_single(recv, send, recv_l, send_l)
        dist.all_to_all_single(back, recv, send_l, recv_l)

    t_f, t_n = _timeit(fused), _timeit(nccl)
    cross = sum(s for r, s in enumerate(send_l) if r != me) * H * 2  # bytes leaving this GPU, each way
    cross = max(cross, sum(s for r, s in enumerate(recv_l) if r != me) * H * 2)
    t_roof = 2 * cross / (LINK_GBS * 1e9) * 1e3  # dispatch + combine
    torch.cuda.synchronize()
    dist.barrier()  # no peer still stores into these buffers
    for x in ex:
        x.close()
    dist.barrier()
    return {"path": f"EP dispatch+combine T={T} H={H} E={E} k={k}", "fused_ms": t_f, "nccl_ms": t_n,
            "roofline_ms": t_roof, "frac": t_roof / t_f}


def bench_dp(numel: int = 256 << 20) -> dict:
    from rl_b200.ops._ext import ext
    from rl_b200.ops.optim import adamw_step
    from rl_b200.parallel.symm import SymmetricBuffer

    n, me = dist.get_world_size(), dist.get_rank()
    grads = SymmetricBuffer(numel * 4)
    params = SymmetricBuffer(numel * 2)
    gv = grads.local_view(torch.float32, numel)
    gv.normal_()
    params.local_view(torch.bfloat16, numel).zero_()
    shard = numel // n
    lo = me * shard
    gshard = torch.empty(shard, device="cuda")
    master = torch.randn(shard, device="cuda")
    m1, m2 = torch.zeros(shard, device="cuda"), torch.zeros(shard, device="cuda")
    nodecay = torch.tensor([[shard, shard]], dtype=torch.int64, device="cuda")
    fence = torch.zeros(1, device="cuda")

    def fused():
        dist.all_reduce(fence)  # peers' gradients complete (as in the optimizer step)
        ext().dp_reduce_shard(grads.ptrs, lo, shard, gshard)
        ext().dp_adam_allgather(params.ptrs, lo, master, gshard, m1, m2, nodecay, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1, 1.0)
        dist.all_reduce(fence)  # every rank's stores landed before the parameters are read

    flat_g = torch.randn(numel, device="cuda")
    flat_p = torch.zeros(numel, dtype=torch.bfloat16, device="cuda")
    pshard = torch.empty(shard, dtype=torch.bfloat16, device="cuda")

    def nccl():
        dist.reduce_scatter_tensor(gshard, flat_g)
        adamw_step(master, gshard, m1, m2, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1, grad_scale=1.0, param_out=pshard)
        dist.all_gather_into_tensor(flat_p, pshard)

    t_f, t_n = _timeit(fused, reps=5), _timeit(nccl, reps=5)
    cross = (n - 1) * shard * 4 + (n - 1) * shard * 2  # gradient shard pulled + parameter shard pushed, per GPU
    t_roof = cross / (LINK_GBS * 1e9) * 1e3
    grads.close_collective()
    params.close_collective()
    return {"path": f"DP RS + AdamW + AG {numel / 2**20:.0f}M params", "fused_ms": t_f, "nccl_ms": t_n,
            "roofline_ms": t_roof, "frac": t_roof / t_f}


def bench_decode_ar(B: int = 64, H: int = 4096) -> dict:
    from rl_b200.ops.norm import add_rms_norm
    from rl_b200.parallel.fused import DecodeAllReduceNorm

    op = DecodeAllReduceNorm(dist.group.WORLD, B, H)
    g = torch.Generator(device="cuda").manual_seed(dist.get_rank())
    partial = torch.randn(B, H, device="cuda", generator=g).to(torch.bfloat16)
    resid = torch.randn(B, H, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.ones(H, device="cuda", dtype=torch.bfloat16)

    def fused():
        op(partial, resid, w, 1e-5)

    red = partial.clone()

    def nccl():
        red.copy_(partial)
        dist.all_reduce(red)
        add_rms_norm(resid, red, w, 1e-5)

    t_f, t_n = _timeit(fused, reps=50), _timeit(nccl, reps=50)
    torch.cuda.synchronize()
    dist.barrier()
    op.close()
    dist.barrier()
    cross = B * H * 2  # this rank's partial rows to the peer
    return {"path": f"TP decode AR + add + RMSNorm B={B} H={H}", "fused_ms": t_f, "nccl_ms": t_n,
            "roofline_ms": cross / (LINK_GBS * 1e9) * 1e3, "frac": cross / (LINK_GBS * 1e9) * 1e3 / t_f}


def main() -> None:
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    rows = []
    for fn in (bench_ep, bench_dp, bench_decode_ar):
        rows.append(fn())
        torch.cuda.synchronize()
        dist.barrier()
    if dist.get_rank() == 0:
        for r in rows:
            print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
