"""Fused compute + collective kernels on 2+ GPUs (NCCL process group, one rank per GPU):
checked against the library baseline (local GEMM, then NCCL reduce-scatter)."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need_gpus(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def case_gemm_rs(rank: int, shapes, iters: int):
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from rl_b200.ops import _ext
    from rl_b200.parallel.fused import GemmReduceScatter

    n = dist.get_world_size()
    op = GemmReduceScatter(dist.group.WORLD, max_rows=max(s[0] for s in shapes), n_cols=max(s[1] for s in shapes))
    errs = []
    for it in range(iters):
        for M, N, K in shapes:
            if N != op.N:
                continue
            g = torch.Generator(device="cuda").manual_seed(1000 * it + rank)
            a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
            w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
            out = op(a, w)
            full = (a.float() @ w.float().t()).to(torch.bfloat16)
            ref = torch.empty(M // n, N, device="cuda", dtype=torch.bfloat16)
            dist.reduce_scatter_tensor(ref, full)
            torch.cuda.synchronize()
            errs.append(((out.float() - ref.float()).norm() / ref.float().norm()).item())
    flag = _ext.ext().gemm_error_flag(True)
    # timing vs the NCCL baseline on the largest shape
    M, N, K = shapes[-1]
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    ref = torch.empty(M // n, N, device="cuda", dtype=torch.bfloat16)

    def timeit(fn, reps=10):
        for _ in range(3):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    t_fused = timeit(lambda: op(a, w))
    t_base = timeit(lambda: dist.reduce_scatter_tensor(ref, torch.matmul(a, w.t())))
    op.close()
    dist.barrier()
    dist.destroy_process_group()
    return {"errs": errs, "flag": flag, "t_fused_ms": t_fused, "t_nccl_ms": t_base, "shape": (M, N, K)}


def test_gemm_reduce_scatter_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    shapes = [(512, 4096, 1024), (2048, 4096, 2048), (1024, 4096, 512), (8192, 4096, 7168)]
    outs = spawn_ranks(case_gemm_rs, 2, shapes, 3, timeout_s=400)
    for o in outs:
        assert o["flag"] == 0
        assert max(o["errs"]) < 2e-2, o["errs"]
    print("gemm_rs timing (max over ranks):", outs[0]["shape"], f"fused {outs[0]['t_fused_ms']:.3f} ms",
          f"cuBLAS+NCCL {outs[0]['t_nccl_ms']:.3f} ms")


def case_tp_sp_model(rank: int, T: int):
    """TP=2 + SP transformer: the fused GEMM + reduce-scatter row-parallel path
    against GEMM then NCCL reduce-scatter (forward output and weight gradients)."""
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.ops import _ext
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(tp=2, backend="nccl", timeout_s=120)
    cfg = ModelConfig(name="tp-sp", vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=4,
                      head_dim=64, ffn_hidden_size=1024, rope_theta=10000.0, max_position_embeddings=1024)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).cuda()
    lens = [T // 2 - 64, T // 2 + 64]
    pos = torch.cat([torch.arange(n) for n in lens]).cuda()
    cu = torch.tensor([0, lens[0], T], dtype=torch.int32).cuda()
    proj = torch.randn(T // 2, cfg.hidden_size, generator=g).cuda()
    res = {}
    for fused in (False, True):
        m = TransformerLM(cfg, ps, seed=5, sequence_parallel=True)
        m.fused_collectives = fused
        h = m(ids, pos, cu, max(lens))
        (h.float() * proj).sum().backward()
        torch.cuda.synchronize()
        grads = {n: p.grad.float().clone() for n, p in m._params.items() if p.grad is not None}
        res[fused] = (h.float().clone(), grads, m._fused_rs is not None and m._fused_ag is not None)
        for op in (m._fused_rs, m._fused_ag):
            if op is not None:
                op.close()
    h0, g0, _ = res[False]
    h1, g1, used = res[True]
    errs = {"hidden": ((h1 - h0).norm() / h0.norm()).item()}
    for n in g0:
        if n in g1:
            errs[n] = ((g1[n] - g0[n]).norm() / (g0[n].norm() + 1e-12)).item()
    flag = _ext.ext().gemm_error_flag(True)
    dist.barrier()
    dist.destroy_process_group()
    return {"errs": errs, "used": used, "flag": flag, "missing": sorted(set(g0) - set(g1))}


def test_tp_sp_model_fused_rs_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_tp_sp_model, 2, 1024, timeout_s=300)
    for o in outs:
        assert o["used"], "fused GEMM+RS / AG+GEMM paths were not taken"
        assert o["flag"] == 0
        assert not o["missing"], o["missing"]
        worst = max(o["errs"].items(), key=lambda kv: kv[1])
        assert worst[1] < 3e-2, worst


def case_refit_reshard(rank: int):
    """Training TP=2 -> rollout TP=1 on 2 GPUs through the native reshard kernels
    (peer loads of the TP partner's flat parameters), bf16 copy and fused fp8
    block quantisation, against torch references built from NCCL-gathered shards."""
    import os
    import time

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.ops import _ext
    from rl_b200.ops.quant import dequant_fp8_block, quant_fp8_block_ref
    from rl_b200.parallel.state import init_distributed
    from rl_b200.weight_sync.reshard import apply_regions_reference

    ps = init_distributed(tp=2, backend="nccl", timeout_s=120)
    cfg = ModelConfig(name="refit", vocab_size=2048, hidden_size=1024, num_layers=2, num_heads=8, num_kv_heads=4,
                      head_dim=128, ffn_hidden_size=2048, rope_theta=10000.0, max_position_embeddings=512)
    pcfg = {"max_total_sequence_length": 128, "precision": "bfloat16",
            "generation": {"temperature": 1.0, "max_new_tokens": 8, "tensor_parallel_size": 1,
                           "vllm_cfg": {"precision": "fp8"}}}
    w = PolicyWorker(pcfg, model_cfg=cfg, pstate=ps, seed=11)
    ws = w.weight_sync
    launches0 = _ext.launch_count()
    with torch.no_grad():
        w.model.flat_param.add_(0.01 * (rank + 1))  # make the shards differ from init
    ws.sync()
    torch.cuda.synchronize()
    launches = _ext.launch_count() - launches0
    src = w.model.flat_param.detach()
    shards = [torch.empty_like(src) for _ in range(2)]
    dist.all_gather(shards, src)
    ref = torch.zeros_like(w.gen_model.flat_param)
    apply_regions_reference(ws.regions, shards, ref)
    copy_err = (ref.float() - w.gen_model.flat_param.float()).abs().max().item()
    q_mismatch, deq_err, scale_err = 0.0, 0.0, 0.0
    for name in ws.q_layout:
        q, s = ws.fp8_weight(name)
        wt = w.gen_model.param(name).detach()
        qr, sr = quant_fp8_block_ref(wt, 128, w.fp8_pow2)  # same scale rule as the worker (pow2 by default)
        # torch divides by the Python scalar 448 through a reciprocal multiply, so its
        # scales may sit one ulp from amax / 448; the bytes are checked against the
        # kernel's own scales (x / s, IEEE division on both sides)
        scale_err = max(scale_err, ((s - sr).abs() / sr).max().item())
        R, C = wt.shape
        full_s = s.repeat_interleave(128, 0)[:R].repeat_interleave(128, 1)[:, :C]
        qk = (wt.float() / full_s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
        q_mismatch = max(q_mismatch, (q.view(torch.uint8) != qk.view(torch.uint8)).float().mean().item())
        a, b = dequant_fp8_block(q, s), dequant_fp8_block(qr, sr)
        deq_err = max(deq_err, ((a - b).abs().max() / b.abs().max()).item())
    # timing (max over ranks)
    for _ in range(3):
        ws.sync()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    reps = 5
    for _ in range(reps):
        ws.sync()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    w.shutdown()
    dist.barrier()
    dist.destroy_process_group()
    return {"copy_err": copy_err, "q_mismatch": q_mismatch, "deq_err": deq_err, "scale_err": scale_err,
            "launches": launches, "ms": t.item(), "bytes": int(w.gen_model.flat_param.numel() * 2)}


def test_refit_reshard_tp2_to_tp1_fp8_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_refit_reshard, 2, timeout_s=300)
    for o in outs:
        assert o["copy_err"] == 0.0, o
        assert o["scale_err"] < 3e-7, o
        assert o["q_mismatch"] == 0.0 and o["deq_err"] < 0.075, o
        assert o["launches"] == 2, o
    print("refit reshard (bf16 copy + fp8 quant):", f"{outs[0]['ms']:.3f} ms for {outs[0]['bytes'] / 2**20:.1f} MiB")


def case_fused_dp_optimizer(rank: int, fused: bool, overlap: bool = False):
    """DP=2 training steps with the fused reduce-scatter / AdamW+all-gather
    kernels (peer loads and stores) or with NCCL; returns what must agree."""
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.ops import _ext
    from rl_b200.parallel.state import init_distributed
    from tests.dist_cases import make_batch

    ps = init_distributed(tp=1, backend="nccl", timeout_s=120)
    cfg = ModelConfig(name="dp", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=64, ffn_hidden_size=512, rope_theta=10000.0, max_position_embeddings=256)
    pcfg = {"max_total_sequence_length": 32, "precision": "bfloat16", "train_global_batch_size": 8,
            "optimizer": {"kwargs": {"lr": 1e-3, "weight_decay": 0.01}},
            "megatron_cfg": {"fused_dp_optimizer": fused,
                             "distributed_data_parallel_config": {"overlap_grad_reduce": overlap}},
            "generation": {"temperature": 1.0, "max_new_tokens": 4},
            "sequence_packing": {"train_mb_tokens": 64, "logprob_mb_tokens": 64}}
    w = PolicyWorker(pcfg, model_cfg=cfg, pstate=ps, seed=3)
    used = w.optimizer._fused(w.optimizer.segments[0])
    if overlap:
        used = used and w._overlap_grad_reduce
    full = make_batch(B=8, S=24, vocab=512, seed=1)
    shard = full.slice(rank * 4, rank * 4 + 4)
    lf = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    res = [w.train(shard, lf, gbs=4) for _ in range(3)]
    torch.cuda.synchronize()
    buckets = sorted(w.optimizer._ov["done"]) if overlap else []
    _ext.check_device_errors()
    flat = w.model.flat_param.float().cpu()
    other = [torch.empty_like(w.model.flat_param) for _ in range(2)]
    dist.all_gather(other, w.model.flat_param)
    same = torch.equal(other[0], other[1])
    w.shutdown()
    dist.barrier()
    dist.destroy_process_group()
    return {"used": used, "loss": [r["loss"] for r in res], "gn": [r["grad_norm"] for r in res], "flat": flat,
            "same": same, "buckets": buckets}


def test_fused_dp_optimizer_matches_nccl_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    a = spawn_ranks(case_fused_dp_optimizer, 2, True, timeout_s=300)
    b = spawn_ranks(case_fused_dp_optimizer, 2, False, timeout_s=300)
    assert a[0]["used"] and not b[0]["used"]
    for x, y in zip(a, b):
        assert x["same"] and y["same"]  # every DP rank holds the same parameters after the all-gather
        for la, lb in zip(x["loss"], y["loss"]):
            assert abs(la - lb) < 1e-3 * max(1.0, abs(lb)), (x["loss"], y["loss"])
        for ga, gb in zip(x["gn"], y["gn"]):
            assert abs(ga - gb) < 1e-3 * max(1.0, gb), (x["gn"], y["gn"])
        d = (x["flat"] - y["flat"]).abs().max().item()
        assert d < 2e-2, d


def test_overlapped_dp_grad_reduce_2gpu():
    """overlap_grad_reduce: per-layer peer-load reductions launched on a side
    stream during the last micro-batch's backward give the parameters of the
    reduction after the backward."""
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    a = spawn_ranks(case_fused_dp_optimizer, 2, True, True, timeout_s=300)
    b = spawn_ranks(case_fused_dp_optimizer, 2, True, False, timeout_s=300)
    for x, y in zip(a, b):
        assert x["used"] and x["same"] and x["buckets"] == [0, 1], x["buckets"]
        assert x["loss"][0] == y["loss"][0] and x["gn"][0] == pytest.approx(y["gn"][0], rel=1e-5)
        for la, lb in zip(x["loss"], y["loss"]):  # later steps: norm partials summed in another grouping
            assert abs(la - lb) < 1e-3 * max(1.0, abs(lb)), (x["loss"], y["loss"])
        d = (x["flat"] - y["flat"]).abs().max().item()
        assert d < 2e-3, d


def case_ag_gemm(rank: int, shapes, iters: int):
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
    from rl_b200.ops import _ext
    from rl_b200.parallel.fused import AllGatherGemm

    n = dist.get_world_size()
    K = shapes[0][2]
    op = AllGatherGemm(dist.group.WORLD, max_rows=max(s[0] for s in shapes), k=K)
    errs = []
    for it in range(iters):
        for M, N, _ in shapes:
            g = torch.Generator(device="cuda").manual_seed(77 * it + rank)
            x = torch.randn(M // n, K, device="cuda", generator=g).to(torch.bfloat16)
            gw = torch.Generator(device="cuda").manual_seed(5 + it)
            w = (torch.randn(N, K, device="cuda", generator=gw) * 0.05).to(torch.bfloat16)
            y, _ = op(x, w)
            full = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
            dist.all_gather_into_tensor(full, x)
            ref = full.float() @ w.float().t()
            torch.cuda.synchronize()
            errs.append(((y.float() - ref).norm() / ref.norm()).item())
    flag = _ext.ext().gemm_error_flag(True)
    M, N, _ = shapes[-1]
    x = torch.randn(M // n, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    full = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)

    def timeit(fn, reps=10):
        for _ in range(3):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    t_fused = timeit(lambda: op(x, w))

    def base():
        dist.all_gather_into_tensor(full, x)
        return torch.matmul(full, w.t())

    t_base = timeit(base)
    op.close()
    dist.barrier()
    dist.destroy_process_group()
    return {"errs": errs, "flag": flag, "t_fused_ms": t_fused, "t_nccl_ms": t_base, "shape": (M, N, K)}


def test_ag_gemm_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    shapes = [(512, 1024, 4096), (2048, 3072, 4096), (16384, 3072, 4096)]
    outs = spawn_ranks(case_ag_gemm, 2, shapes, 3, timeout_s=400)
    for o in outs:
        assert o["flag"] == 0
        assert max(o["errs"]) < 2e-2, o["errs"]
    print("ag_gemm timing (max over ranks):", outs[0]["shape"], f"fused {outs[0]['t_fused_ms']:.3f} ms",
          f"NCCL+cuBLAS {outs[0]['t_nccl_ms']:.3f} ms")


def case_ep_moe(rank: int, T: int):
    """EP=2 MoE transformer: peer-store dispatch / combine kernels against the
    NCCL all-to-all path (forward output and gradients, two steps so both
    epoch parities of the exchange buffers are used)."""
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.ops import _ext
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(ep=2, backend="nccl", timeout_s=120)
    cfg = ModelConfig(name="ep", vocab_size=1024, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=64, ffn_hidden_size=0, rope_theta=10000.0, qk_norm=True, num_experts=8, moe_top_k=2,
                      moe_ffn_hidden_size=128, moe_aux_loss_coef=0.0, max_position_embeddings=1024)
    g = torch.Generator().manual_seed(11 + rank)  # ranks hold different tokens
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).cuda()
    lens = [T // 2, T - T // 2]
    pos = torch.cat([torch.arange(n) for n in lens]).cuda()
    cu = torch.tensor([0, lens[0], T], dtype=torch.int32).cuda()
    proj = torch.randn(T, cfg.hidden_size, generator=g).cuda()
    res = {}
    for fused in (False, True):
        m = TransformerLM(cfg, ps, seed=5)
        m.fused_collectives = fused
        hs, grads = [], None
        for _ in range(2):
            h = m(ids, pos, cu, max(lens))
            (h.float() * proj).sum().backward()
            hs.append(h.float().clone())
        torch.cuda.synchronize()
        grads = {n: p.grad.float().clone() for n, p in m._params.items() if p.grad is not None}
        res[fused] = (hs, grads, m._ep_ex is not None)
        if m._ep_ex is not None:
            for x in m._ep_ex:
                x.close()
    errs = {}
    for j in range(2):
        errs[f"hidden{j}"] = ((res[True][0][j] - res[False][0][j]).norm() / res[False][0][j].norm()).item()
    for n_, g0 in res[False][1].items():
        if n_ in res[True][1]:
            errs[n_] = ((res[True][1][n_] - g0).norm() / (g0.norm() + 1e-12)).item()
    flag = _ext.ext().ep_error_flag(True)
    dist.barrier()
    dist.destroy_process_group()
    return {"errs": errs, "used": res[True][2], "flag": flag, "missing": sorted(set(res[False][1]) - set(res[True][1]))}


def test_ep_moe_fused_dispatch_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_ep_moe, 2, 384, timeout_s=300)
    for o in outs:
        assert o["used"], "fused EP exchange was not taken"
        assert o["flag"] == 0
        assert not o["missing"], o["missing"]
        worst = max(o["errs"].items(), key=lambda kv: kv[1])
        assert worst[1] < 3e-2, worst


def case_cp_model(rank: int):
    """CP=2 transformer on 2 GPUs: the overlapped K/V exchange (copy-engine pulls +
    per-block flag waits in the attention kernel) against the NCCL all-gather
    path (forward output and gradients)."""
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.ops import _ext
    from rl_b200.parallel.context_parallel import cp_layout
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(cp=2, backend="nccl", timeout_s=120)
    cfg = ModelConfig(name="cp", vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=4,
                      head_dim=64, ffn_hidden_size=1024, rope_theta=10000.0, max_position_embeddings=4096)
    lens = [700, 1500, 256]
    lay = cp_layout(lens, 2, ps.cp_rank, torch.device("cuda"), unit=64)
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (lay.T_local,), generator=torch.Generator().manual_seed(3 + rank)).cuda()
    proj = torch.randn(lay.T_local, cfg.hidden_size, generator=g).cuda()
    res = {}
    for fused in (False, True):
        m = TransformerLM(cfg, ps, seed=5)
        m.fused_collectives = fused
        m._cp_layout = lay
        hs = []
        for _ in range(2):
            h = m(ids, lay.positions, None, lay.max_k)
            (h.float() * proj).sum().backward()
            hs.append(h.float().clone())
        torch.cuda.synchronize()
        grads = {n: p.grad.float().clone() for n, p in m._params.items() if p.grad is not None}
        res[fused] = (hs, grads, m._cp_ex is not None)
        if m._cp_ex is not None:
            m._cp_ex.close()
    errs = {f"hidden{j}": ((res[True][0][j] - res[False][0][j]).norm() / res[False][0][j].norm()).item()
            for j in range(2)}
    for n_, g0 in res[False][1].items():
        if n_ in res[True][1]:
            errs[n_] = ((res[True][1][n_] - g0).norm() / (g0.norm() + 1e-12)).item()
    flag = _ext.ext().attn_error_flag(True)
    dist.barrier()
    dist.destroy_process_group()
    return {"errs": errs, "used": res[True][2], "flag": flag}


def test_cp_overlapped_kv_exchange_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_cp_model, 2, timeout_s=300)
    for o in outs:
        assert o["used"], "overlapped CP exchange was not taken"
        assert o["flag"] == 0
        worst = max(o["errs"].items(), key=lambda kv: kv[1])
        assert worst[1] < 3e-2, worst


def case_decode_ar(rank: int):
    """TP=2 decode step: fused peer-memory all-reduce + residual add + RMSNorm
    against NCCL all-reduce + add_rms_norm, three calls in a row and once more
    under CUDA-graph replay."""
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import KVCache, TransformerLM
    from rl_b200.ops import _ext
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(tp=2, backend="nccl", timeout_s=120)
    cfg = ModelConfig(name="dar", vocab_size=1024, hidden_size=512, num_layers=3, num_heads=8, num_kv_heads=4,
                      head_dim=64, ffn_hidden_size=1024, rope_theta=10000.0, max_position_embeddings=512)
    B, bs = 48, 16
    m = TransformerLM(cfg, ps, seed=5)
    kv = KVCache(cfg.num_layers, B * 4 + 1, bs, m.nkv, m.hd, torch.bfloat16, torch.device("cuda"))
    bt = (torch.arange(B * 4, dtype=torch.int32).view(B, 4) + 1).cuda()
    outs = {}
    for fused in (False, True):
        m.fused_collectives = fused
        res = []
        for step in range(3):
            g = torch.Generator().manual_seed(step)
            tok = torch.randint(0, cfg.vocab_size, (B,), generator=g).cuda()
            pos = torch.full((B,), step, dtype=torch.int32, device="cuda")
            slot = bt[:, 0].long() * bs + step
            res.append(m.forward_decode(tok, pos, kv, bt, pos + 1, slot, 64).float().clone())
        outs[fused] = res
    # graph replay of the fused step
    tok = torch.randint(0, cfg.vocab_size, (B,), generator=torch.Generator().manual_seed(9)).cuda()
    pos = torch.full((B,), 3, dtype=torch.int32, device="cuda")
    slot = bt[:, 0].long() * bs + 3
    eager = m.forward_decode(tok, pos, kv, bt, pos + 1, slot, 64).float().clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        m.forward_decode(tok, pos, kv, bt, pos + 1, slot, 64)
    torch.cuda.current_stream().wait_stream(s)
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph):
        y = m.forward_decode(tok, pos, kv, bt, pos + 1, slot, 64)
    replays = []
    for _ in range(2):
        gph.replay()
        torch.cuda.synchronize()
        replays.append(y.float().clone())
    errs = [((a - b).norm() / b.norm()).item() for a, b in zip(outs[True], outs[False])]
    errs += [((r - eager).norm() / eager.norm()).item() for r in replays]
    flag = _ext.ext().decode_ar_error_flag(True)
    del gph
    m._decode_ar.close()
    dist.barrier()
    dist.destroy_process_group()
    return {"errs": errs, "flag": flag}


def test_decode_allreduce_rmsnorm_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_decode_ar, 2, timeout_s=300)
    for o in outs:
        assert o["flag"] == 0
        assert max(o["errs"]) < 1e-2, o["errs"]


def case_pp_train(rank: int, big: bool = False, vpp: int = 1):
    """PP=2 on 2 GPUs (NCCL send / recv between the stages, 1F1B schedule): one
    GRPO-loss training step and the log-probs after it against a single-GPU
    worker of the same seed on the same batch.  ``big`` makes every activation
    message 16 MiB, above NCCL's 4 MiB channel buffer, so a send finishes only
    once its receive runs; ``vpp`` > 1 runs the interleaved schedule."""
    import os

    import torch.distributed as dist

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed, single_process_state
    from tests.dist_cases import make_batch

    ps = init_distributed(pp=2, backend="nccl", timeout_s=120)
    H, mb = (2048, 4096) if big else (512, 512)
    cfg = ModelConfig(name="pp", vocab_size=1024, hidden_size=H, num_layers=4, num_heads=8, num_kv_heads=4,
                      head_dim=H // 8, ffn_hidden_size=2 * H, rope_theta=10000.0, max_position_embeddings=1024)
    pcfg = {"max_total_sequence_length": 256, "precision": "bfloat16",
            "optimizer": {"kwargs": {"lr": 1e-4, "weight_decay": 0.01}},
            "generation": {"temperature": 1.0, "max_new_tokens": 4},
            "megatron_cfg": {"virtual_pipeline_model_parallel_size": vpp} if vpp > 1 else {},
            "sequence_packing": {"train_mb_tokens": mb, "logprob_mb_tokens": mb}}
    batch = make_batch(B=64 if big else 16, S=256 if big else 200, vocab=1024)
    loss_fn = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    w = PolicyWorker(pcfg, model_cfg=cfg, pstate=ps, seed=11)
    res = w.train(batch, loss_fn, gbs=batch.size)
    lp = w.get_logprobs(batch)["logprobs"]
    w.shutdown()
    ref = PolicyWorker(pcfg, model_cfg=cfg, pstate=single_process_state(torch.device("cuda", rank)), seed=11)
    res1 = ref.train(batch, loss_fn, gbs=batch.size)
    lp1 = ref.get_logprobs(batch)["logprobs"]
    ref.shutdown()
    mask = batch["token_mask"] > 0
    out = {"loss": (res["loss"], res1["loss"]), "gn": (res["grad_norm"], res1["grad_norm"]),
           "lp_err": (lp - lp1)[mask].abs().max().item(), "stage_layers": list(w.model.layer_range)}
    dist.barrier()
    dist.destroy_process_group()
    return out


def test_pipeline_parallel_train_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_pp_train, 2, timeout_s=300)
    assert outs[0]["stage_layers"] == [0, 1] and outs[1]["stage_layers"] == [2, 3]
    for o in outs:
        (a, b), (g, h) = o["loss"], o["gn"]
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), o
        assert abs(g - h) < 3e-2 * h, o
        assert o["lp_err"] < 0.15, o


@pytest.mark.skip(reason="16 MiB stage messages on two B200s stopped progressing within the test's limit; the same "
                         "schedule over gloo completes; cause not found")
@pytest.mark.parametrize("vpp", [1, 2])
def test_pipeline_parallel_large_messages_2gpu(vpp):
    """16 MiB activations (above NCCL's channel buffer) through 1F1B and the
    interleaved schedule finish within the process-group timeout and match the
    single-GPU step."""
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_pp_train, 2, True, vpp, timeout_s=300)
    for o in outs:
        (a, b), (g, h) = o["loss"], o["gn"]
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), o
        assert abs(g - h) < 3e-2 * h, o
        assert o["lp_err"] < 0.15, o


def _ce_policy(q_meta, q_done, dev):
    import torch

    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.weight_sync.checkpoint_engine import CheckpointEngineSynchronizer, create_checkpoint_engine

    torch.cuda.set_device(dev)
    cfg = ModelConfig(name="ce", vocab_size=1024, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=64, ffn_hidden_size=512, rope_theta=10000.0, max_position_embeddings=256)
    eng = create_checkpoint_engine("cuda_ipc", bucket_size_bytes=1 << 18,
                                   engine_kwargs={"is_master": True, "port": 0, "timeout_s": 120})
    meta = eng.prepare()
    eng.init_policy_process_group(worker_rank=0, train_world_size=1, rollout_world_size=1, metadata=[meta])
    q_meta.put((meta, eng.port))
    m = TransformerLM(cfg, device=torch.device("cuda", dev), dtype=torch.bfloat16, seed=3)
    sync = CheckpointEngineSynchronizer(eng, m)
    sync.sync()
    q_done.get(timeout=120)
    eng.close()


def _ce_rollout(meta, port, q_out, dev):
    import torch

    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.weight_sync.checkpoint_engine import CheckpointEngineSynchronizer, create_checkpoint_engine

    torch.cuda.set_device(dev)
    cfg = ModelConfig(name="ce", vocab_size=1024, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=64, ffn_hidden_size=512, rope_theta=10000.0, max_position_embeddings=256)
    eng = create_checkpoint_engine("cuda_ipc", bucket_size_bytes=1 << 18, engine_kwargs={"port": port,
                                                                                          "timeout_s": 120})
    eng.init_rollout_process_group(rollout_rank=0, train_world_size=1, rollout_world_size=1, metadata=[meta])
    m = TransformerLM(cfg, device=torch.device("cuda", dev), dtype=torch.bfloat16, seed=77)
    ref = TransformerLM(cfg, device=torch.device("cuda", dev), dtype=torch.bfloat16, seed=3)
    n = CheckpointEngineSynchronizer(eng, m).receive_into(m)
    q_out.put((n, bool(torch.equal(m.flat_param, ref.flat_param)), eng.seq))
    eng.close()


def test_cuda_ipc_checkpoint_engine_2gpu():
    """Refit between two processes with no process group: the policy's weights
    leave through two CUDA IPC slots in its HBM and land on the other GPU."""
    _need_gpus(2)
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_meta, q_done, q_out = ctx.Queue(), ctx.Queue(), ctx.Queue()
    pp = ctx.Process(target=_ce_policy, args=(q_meta, q_done, 0))
    pp.start()
    meta, port = q_meta.get(timeout=180)
    rp = ctx.Process(target=_ce_rollout, args=(meta, port, q_out, 1))
    rp.start()
    try:
        n, same, buckets = q_out.get(timeout=240)
    finally:
        q_done.put(True)
        rp.join(60)
        pp.join(60)
    assert same and n > 0 and buckets > 4


def case_nvls(rank: int):
    """NVLS multicast all-reduce / reduce-scatter kernels against NCCL, plus a
    timing of both on a 256 MiB fp32 buffer (events, max over ranks)."""
    import gc

    import torch.distributed as dist

    from datetime import timedelta

    torch.cuda.set_device(rank)
    # a short timeout: a rank that fell out of step ends the test instead of hanging it
    dist.init_process_group("nccl", device_id=torch.device("cuda", rank), timeout=timedelta(seconds=60))
    from rl_b200.ops._ext import ext

    res, bufs = {}, []
    ok = torch.ones(1, device="cuda")
    try:
        from rl_b200.parallel.nvls import NVLSBuffer

        bufs = [NVLSBuffer(1 << 20, torch.float32), NVLSBuffer(1 << 20, torch.bfloat16),
                NVLSBuffer(64 << 20, torch.float32)]
    except Exception as e:  # noqa: BLE001 - reported; every rank then skips the NVLS calls together
        res["unavailable"] = repr(e)
        ok.zero_()
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() == 1:
        n = dist.get_world_size()
        g = torch.Generator(device="cuda").manual_seed(rank)
        for b, key in ((bufs[0], "f32"), (bufs[1], "bf16")):
            x = torch.randn(b.tensor.numel(), device="cuda", generator=g).to(b.tensor.dtype)
            b.tensor.copy_(x)
            ref = x.clone()
            dist.all_reduce(ref)
            b.all_reduce_()
            torch.cuda.synchronize()
            res[key + "_err"] = (b.tensor.float() - ref.float()).abs().max().item()
        # reduce-scatter: each rank sums its own half
        x = torch.randn(1 << 20, device="cuda", generator=g)
        bufs[0].tensor.copy_(x)
        full = x.clone()
        dist.all_reduce(full)
        per = (1 << 20) // n
        out = torch.empty(per, device="cuda")
        bufs[0].reduce_shard(rank * per, per, out)
        torch.cuda.synchronize()
        res["rs_err"] = (out - full[rank * per:(rank + 1) * per]).abs().max().item()
        big = bufs[2]
        big.tensor.normal_()
        ref = torch.randn(64 << 20, device="cuda")

        def timeit(fn, reps=10):
            for _ in range(3):
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
            return t.item()

        res["t_nvls_ms"] = timeit(big.all_reduce_)
        res["t_nccl_ms"] = timeit(lambda: dist.all_reduce(ref))
        res["flag"] = int(ext().nvls_error_flag(True))
    torch.cuda.synchronize()
    dist.barrier()
    del bufs
    gc.collect()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    return res


def test_nvls_multicast_collectives_2gpu():
    _need_gpus(2)
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(case_nvls, 2, timeout_s=300)
    if "unavailable" in outs[0]:
        pytest.skip(outs[0]["unavailable"])
    for o in outs:
        assert o["flag"] == 0
        assert o["f32_err"] < 1e-5 and o["rs_err"] < 1e-5, o
        assert o["bf16_err"] < 0.05, o
    nb = 64 * 4 * 2**20
    print("NVLS all-reduce 256 MiB fp32:", f"{outs[0]['t_nvls_ms']:.3f} ms", f"(bus {2 * nb / 2 / outs[0]['t_nvls_ms'] / 1e6:.0f} GB/s)",
          f"NCCL {outs[0]['t_nccl_ms']:.3f} ms")
