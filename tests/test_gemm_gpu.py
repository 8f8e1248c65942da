"""The general tcgen05 GEMM (``csrc/gemm_sm100.cu``) against an fp32 PyTorch
product: every operand-major combination a linear layer uses (forward NT, input
gradient NN, weight gradient TN), both tile shapes (1-CTA 128x256, 2-CTA
256x256), ragged M / N / K, and the bf16, fp32 and fp32-accumulate epilogues."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(256, 256, 64), (1000, 1000, 200), (384, 776, 1088), (2048, 1536, 4096)]


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _operands(M, N, K, a_mn, b_mn, dev, g):
    a = torch.randn(*((K, M) if a_mn else (M, K)), device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn(*((K, N) if b_mn else (N, K)), device=dev, generator=g).to(torch.bfloat16)
    af = a.float().t() if a_mn else a.float()
    bf = b.float() if b_mn else b.float().t()
    return a, b, af @ bf  # fp32 reference [M, N]


@pytest.mark.parametrize("tile", [1, 2])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_sm100_bf16_out(cuda_device, tile, a_mn, b_mn):
    from rl_b200.ops._ext import ext

    C = ext()
    g = torch.Generator(device=cuda_device).manual_seed(7)
    for M, N, K in SHAPES:
        a, b, ref = _operands(M, N, K, a_mn, b_mn, cuda_device, g)
        out = torch.full((M, N), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        C.gemm_sm100(a, b, out, a_mn, b_mn, False, tile)
        torch.cuda.synchronize()
        assert C.gemm_sm100_error_flag(True) == 0
        assert _rel(out, ref) < 1e-2, (M, N, K, _rel(out, ref))


@pytest.mark.parametrize("tile", [1, 2])
def test_gemm_sm100_fp32_accumulate(cuda_device, tile):
    """Weight-gradient form: main_grad (fp32) += dy^T x, twice in a row."""
    from rl_b200.ops._ext import ext

    C = ext()
    g = torch.Generator(device=cuda_device).manual_seed(3)
    for M, N, K in SHAPES:
        base = torch.randn(M, N, device=cuda_device, generator=g)
        acc = base.clone()
        want = base.clone()
        for _ in range(2):
            a, b, ref = _operands(M, N, K, True, True, cuda_device, g)
            C.gemm_sm100(a, b, acc, True, True, True, tile)
            want += ref
        torch.cuda.synchronize()
        assert C.gemm_sm100_error_flag(True) == 0
        assert _rel(acc, want) < 1e-5, (M, N, K, _rel(acc, want))
        out = torch.empty(M, N, device=cuda_device)
        a, b, ref = _operands(M, N, K, False, True, cuda_device, g)
        C.gemm_sm100(a, b, out, False, True, False, tile)
        torch.cuda.synchronize()
        assert _rel(out, ref) < 1e-5


def test_gemm_ops_route_to_native(cuda_device):
    """mm_nt / mm_nn / mm_tn / mm_tn_accumulate of rl_b200.ops.gemm match fp32
    products, and every one of them ran the tcgen05 kernel (not the library)."""
    from torch.profiler import ProfilerActivity, profile

    from rl_b200.ops import gemm

    g = torch.Generator(device=cuda_device).manual_seed(1)
    T, N, K = 2048, 4096, 2048
    x = torch.randn(T, K, device=cuda_device, generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, N, device=cuda_device, generator=g).to(torch.bfloat16)
    acc = torch.ones(N, K, device=cuda_device)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        y = gemm.mm_nt(x, w)
        dx = gemm.mm_nn(dy, w)
        dw = gemm.mm_tn(dy, x)
        gemm.mm_tn_accumulate(dy, x, acc)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert sum("gemm_kernel" in n for n in names) == 4, names
    assert _rel(y, x.float() @ w.float().t()) < 1e-2
    assert _rel(dx, dy.float() @ w.float()) < 1e-2
    assert _rel(dw, dy.float().t() @ x.float()) < 1e-2
    assert _rel(acc, 1 + dy.float().t() @ x.float()) < 1e-5
