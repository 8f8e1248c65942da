"""The allocation-free RMSNorm-backward entry point (``rlb_rmsnorm_bwd_noalloc``).

Some callers of this library cannot allocate device memory: code hosted by a
runtime that owns all of the GPU's memory, or paths that must not pay the
implicit synchronisation of cudaMalloc/cudaFree.  For them the library exports a
plain C function whose scratch lives in a fixed device array.  This test calls
it through the exported C symbol (as such a caller would, via ctypes) and
checks it against an fp32 PyTorch RMSNorm backward and against the regular
tensor entry point, on calls in a row (including a hidden size that is not a
multiple of 8), that a call after the first allocates no device memory, and
that a size beyond the static maximum is rejected.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_HIDDEN = 8192  # RLB_NOALLOC_MAX_HIDDEN in csrc/noalloc.h
EPS = 1e-5


def _lib():
    from rl_b200 import _C  # loads the library (and its torch dependencies) into the process

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.rlb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    err = lib.rlb_noalloc_last_error
    err.restype = ctypes.c_char_p
    err.argtypes = []
    return _C, fn, err


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _fp32_reference(dy, x, w):
    """RMSNorm backward in fp32 by autograd: y = x / sqrt(mean(x^2) + eps) * w."""
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS) * wf
    y.backward(dy.float())
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + EPS)
    return xf.grad, wf.grad, rstd


def _call(fn, err, dy, x, w, rstd, dx, dw, stream):
    rows, hidden = x.shape
    rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows,
            hidden, ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, err()


def test_noalloc_rmsnorm_bwd_matches_fp32_reference(cuda_device):
    C, fn, err = _lib()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream()
    # calls in a row with different sizes; 2050 is not a multiple of 8 (the scalar path)
    for rows, hidden in ((300, 4096), (1000, 5120), (257, 2050)):
        x = torch.randn(rows, hidden, device=cuda_device, dtype=torch.bfloat16)
        w = (1 + 0.1 * torch.randn(hidden, device=cuda_device)).to(torch.bfloat16)
        dy = torch.randn(rows, hidden, device=cuda_device, dtype=torch.bfloat16)
        dx_ref, dw_ref, rstd = _fp32_reference(dy, x, w)
        dx = torch.empty_like(x)
        dw = torch.full((hidden,), float("nan"), device=cuda_device)
        _call(fn, err, dy, x, w, rstd, dx, dw, stream)
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 2e-2, (rows, hidden)
        assert _rel(dw, dw_ref) < 1e-2, (rows, hidden)
        # and the same numbers as the tensor entry point (same kernels, allocated scratch)
        dx_t, dw_t = C.rmsnorm_bwd(dy, x, w, rstd)
        assert _rel(dx, dx_t) < 1e-2 and _rel(dw, dw_t) < 1e-3


def test_noalloc_later_calls_allocate_nothing(cuda_device):
    _, fn, err = _lib()
    torch.manual_seed(1)
    stream = torch.cuda.current_stream()
    rows, hidden = 512, 4096
    x = torch.randn(rows, hidden, device=cuda_device, dtype=torch.bfloat16)
    w = torch.ones(hidden, device=cuda_device, dtype=torch.bfloat16)
    dy = torch.randn_like(x)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + EPS)
    dx = torch.empty_like(x)
    dw = torch.empty(hidden, device=cuda_device)
    _call(fn, err, dy, x, w, rstd, dx, dw, stream)  # the first call on the device may load the module
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(3):
        _call(fn, err, dy, x, w, rstd, dx, dw, stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_oversized_hidden(cuda_device):
    _, fn, err = _lib()
    hidden = MAX_HIDDEN + 8
    t = torch.zeros(4, hidden, device=cuda_device, dtype=torch.bfloat16)
    w = torch.ones(hidden, device=cuda_device, dtype=torch.bfloat16)
    r = torch.ones(4, device=cuda_device)
    dw = torch.zeros(hidden, device=cuda_device)
    rc = fn(t.data_ptr(), t.data_ptr(), w.data_ptr(), r.data_ptr(), t.data_ptr(), dw.data_ptr(), 4, hidden, None)
    assert rc != 0
    assert b"exceeds" in err()
