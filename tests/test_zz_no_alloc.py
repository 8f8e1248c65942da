"""The allocation-free RMSNorm-backward entry point (``rlb_rmsnorm_bwd_noalloc``).

Some callers of this library cannot allocate device memory: code hosted by a
runtime that owns all of the GPU's memory, or paths that must not pay the
implicit synchronisation of cudaMalloc/cudaFree.  For them the library exports a
plain C function whose scratch lives in a fixed device array.  This test calls
it through the exported C symbol (as such a caller would, via ctypes) and
checks it against the regular tensor entry point, on two calls in a row, plus
the rejection of a size beyond the static maximum.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_HIDDEN = 8192  # RLB_NOALLOC_MAX_HIDDEN in csrc/noalloc.h


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


def test_noalloc_rmsnorm_bwd_matches_tensor_entry_point(cuda_device):
    C, fn, err = _lib()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream()
    for rows, hidden in ((300, 4096), (1000, 5120)):  # two calls in a row, different sizes
        x = torch.randn(rows, hidden, device=cuda_device, dtype=torch.bfloat16)
        w = (1 + 0.1 * torch.randn(hidden, device=cuda_device)).to(torch.bfloat16)
        dy = torch.randn(rows, hidden, device=cuda_device, dtype=torch.bfloat16)
        _, rstd = C.rmsnorm_fwd(x, w, 1e-5)
        dx_ref, dw_ref = C.rmsnorm_bwd(dy, x, w, rstd)
        dx = torch.empty_like(x)
        dw = torch.full((hidden,), float("nan"), device=cuda_device)
        rc = fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows,
                hidden, ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, err()
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 2e-2
        assert _rel(dw, dw_ref) < 2e-2


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
