"""Race / bounds detection aids on one GPU: guard canaries around symmetric
buffers, and the bounds-checked debug build (``rl_b200._C_debug``) that reports a
data-dependent index outside its tensor instead of dereferencing it.

Every out-of-range index used here points into memory the test owns: the
tensors handed to the kernels are slices of larger allocations (and the canary
write lands inside the buffer's own guard), so even a build without the checks
would touch only owned memory."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_symmetric_buffer_canaries(cuda_device, monkeypatch):
    from rl_b200.ops._ext import DeviceBoundsError, ext
    from rl_b200.parallel import symm

    monkeypatch.setenv("RL_B200_CANARIES", "1")
    b = symm.SymmetricBuffer(1 << 20)
    try:
        assert b.guard == symm.GUARD and b.canary_intact()
        symm.check_canaries()
        body = b.local_view(torch.float32, (1 << 20) // 4)
        body.fill_(3.0)  # writes inside the buffer leave the guards alone
        torch.cuda.synchronize()
        symm.check_canaries()
        # a store 16 floats past the end: inside the tail guard (owned memory)
        over = ext().symm_view(b.local_ptr, (1 << 20) // 4 + 16, 6, b.device)
        over[-1] = 1.0
        torch.cuda.synchronize()
        assert not b.canary_intact()
        with pytest.raises(DeviceBoundsError, match="guard overwritten"):
            symm.check_canaries()
    finally:
        b.close()
    symm.check_canaries()  # closed buffers are no longer checked


_DEBUG_CASE = r"""
import torch
from rl_b200.ops import _ext
from rl_b200.ops._ext import DeviceBoundsError, ext
m = ext()._mod
assert m.__name__.endswith("_C_debug") and m.debug_bounds_build(), m.__name__
dev = torch.device("cuda", 0)
# KV-cache write: 4 tokens, cache of 8 slots carved out of a 16-slot allocation
nkv, hd = 2, 64
parent_k = torch.zeros(16, nkv, hd, device=dev, dtype=torch.bfloat16)
parent_v = torch.zeros_like(parent_k)
kc, vc = parent_k[:8], parent_v[:8]
k = torch.ones(4, nkv, hd, device=dev, dtype=torch.bfloat16)
v = torch.ones_like(k)
slots = torch.tensor([0, 3, 8, 12], device=dev)  # 8 and 12 are past the 8-slot cache
ext().write_kv_cache(k, v, kc, vc, slots, 1.0, 1.0)
torch.cuda.synchronize()
assert float(parent_k[3].sum()) == nkv * hd and float(parent_k[0].sum()) == nkv * hd
assert float(parent_k[8:].abs().sum()) == 0.0, "an out-of-range slot was written"
try:
    _ext.check_device_errors()
    raise SystemExit("no bounds error reported")
except DeviceBoundsError as e:
    assert "KV-cache slot index 8" in str(e) or "KV-cache slot index 12" in str(e), str(e)
_ext.check_device_errors()  # reading cleared the word
# paged decode: block table entry past the cache's blocks (cache carved from a larger one)
bs, nblk = 16, 4
kcache = torch.randn(2 * nblk, bs, nkv, hd, device=dev, dtype=torch.bfloat16)[:nblk]
vcache = torch.randn(2 * nblk, bs, nkv, hd, device=dev, dtype=torch.bfloat16)[:nblk]
q = torch.randn(1, 8, hd, device=dev, dtype=torch.bfloat16)
bt = torch.tensor([[0, 1, 6, 3]], device=dev, dtype=torch.int32)  # 6 >= 4 blocks
sl = torch.tensor([64], device=dev, dtype=torch.int32)
ext().paged_decode_attn(q, kcache, vcache, bt, sl, hd ** -0.5, 0, 1.0, 1.0)
torch.cuda.synchronize()
try:
    _ext.check_device_errors()
    raise SystemExit("no block-table error reported")
except DeviceBoundsError as e:
    assert "block-table entry index 6" in str(e), str(e)
print("debug-bounds ok")
"""


def test_bounds_checked_debug_build_reports_bad_indices(cuda_device):
    if not any(f.startswith("_C_debug") and f.endswith(".so") for f in os.listdir(os.path.join(ROOT, "rl_b200"))):
        pytest.skip("debug build not present (RL_B200_DEBUG_BOUNDS=1 python setup.py build_ext --inplace)")
    env = dict(os.environ, RL_B200_DEBUG_BOUNDS="1")
    r = subprocess.run([sys.executable, "-c", _DEBUG_CASE], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "debug-bounds ok" in r.stdout, r.stdout + r.stderr
