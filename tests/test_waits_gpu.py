"""Bounded in-kernel waits: a flag that nothing ever sets makes the kernel give
up after the configured bound, set its error word and return; the host then
raises, and the CUDA context stays usable (failure detection made testable
without a GPU fault).

The wait exercised here is the context-parallel key-arrival wait of the tcgen05
attention forward: every key block waits for the copy flag of the rank that owns
its chunk.  With the flags left at 0 and a 1 ms bound, the kernel must come back
quickly with error code 5."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_wait_expires_and_host_raises(cuda_device):
    from rl_b200.ops._ext import DeviceWaitError, check_device_errors, ext

    C = ext()
    check_device_errors()  # start clean
    old = C.peer_wait_cycles()
    torch.manual_seed(0)
    q = torch.randn(256, 4, 128, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(512, 2, 128, device=cuda_device).to(torch.bfloat16)
    v = torch.randn(512, 2, 128, device=cuda_device).to(torch.bfloat16)
    seg = torch.tensor([[0, 256, 256, 256]], dtype=torch.int32, device=cuda_device)  # chunk 1 vs keys [256, 512)
    flags = torch.zeros(2, dtype=torch.int32, device=cuda_device)  # never written: no copy will ever land
    try:
        C.set_peer_wait_cycles(2_000_000)  # ~1 ms at B200 clocks
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        C.flash_attn_seg_fwd_tc(q, k, v, seg, 256, 128 ** -0.5, flags, 1, 2)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert dt < 5.0, dt  # returned well before the default ~2 s bound per wait would add up
        assert C.attn_tc_error_flag(False) == 5
        with pytest.raises(DeviceWaitError):
            check_device_errors()
        assert C.attn_tc_error_flag(False) == 0  # cleared by the check
    finally:
        C.set_peer_wait_cycles(old)
    # the context is intact: with the flags set, the same call completes and is correct
    flags.fill_(1)
    o, _ = C.flash_attn_seg_fwd_tc(q, k, v, seg, 256, 128 ** -0.5, flags, 1, 2)
    torch.cuda.synchronize()
    check_device_errors()
    qf = q.float().transpose(0, 1)
    kf = k[256:].float().transpose(0, 1).repeat_interleave(2, 0)
    vf = v[256:].float().transpose(0, 1).repeat_interleave(2, 0)
    sc = (qf @ kf.transpose(-1, -2)) * 128 ** -0.5
    sc = sc.masked_fill(torch.ones(256, 256, device=cuda_device, dtype=torch.bool).triu(1), float("-inf"))
    ref = (torch.softmax(sc, -1) @ vf).transpose(0, 1)
    err = ((o.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err
