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
