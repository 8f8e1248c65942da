"""Numerics of every native sm_100a kernel against a plain PyTorch fp32 reference of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from rl_b200.ops import _ext  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _need_ext(cuda_device):
    assert _ext.has_ext(), "native extension must be built and loadable on a GPU box"
    yield


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def test_rmsnorm_fwd_bwd(cuda_device):
    from rl_b200.ops.norm import add_rms_norm, add_rms_norm_ref, rms_norm, rms_norm_ref

    torch.manual_seed(0)
    for H in (64, 4096, 5120, 100):
        x = torch.randn(37, H, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
        w = (1 + 0.1 * torch.randn(H, device=cuda_device)).to(torch.bfloat16).requires_grad_(True)
        y = rms_norm(x, w, 1e-5)
        xr = x.detach().float().requires_grad_(True)
        wr = w.detach().float().requires_grad_(True)
        yr = rms_norm_ref(xr, wr, 1e-5)
        assert rel_err(y, yr) < 1e-2
        g = torch.randn_like(yr)
        y.backward(g.to(torch.bfloat16))
        yr.backward(g)
        assert rel_err(x.grad, xr.grad) < 2e-2
        assert rel_err(w.grad, wr.grad) < 2e-2
    # fused residual add
    H = 4096
    x = torch.randn(19, H, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    d = torch.randn(19, H, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    w = torch.ones(H, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    y, s = add_rms_norm(x, d, w, 1e-5)
    xr, dr, wr = (t.detach().float().requires_grad_(True) for t in (x, d, w))
    yr, sr = add_rms_norm_ref(xr, dr, wr, 1e-5)
    assert rel_err(y, yr) < 1e-2 and rel_err(s, sr) < 1e-2
    gy, gs = torch.randn_like(yr), torch.randn_like(sr)
    (y.float() * gy + s.float() * gs).sum().backward()
    (yr * gy + sr * gs).sum().backward()
    assert rel_err(x.grad, xr.grad) < 2e-2 and rel_err(d.grad, dr.grad) < 2e-2
    assert rel_err(w.grad, wr.grad) < 2e-2


def test_rope_and_inverse(cuda_device):
    from rl_b200.ops.rope import apply_rope_qkv, apply_rope_qkv_ref, build_rope_cache

    nq, nkv, hd, T = 8, 2, 128, 50
    cache = build_rope_cache(4096, hd, 500000.0, {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                  "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                             device=cuda_device)
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    pos = torch.randint(0, 4000, (T,), device=cuda_device, dtype=torch.int32)
    out = apply_rope_qkv(qkv, pos, cache, nq, nkv, hd)
    ref = apply_rope_qkv_ref(qkv.detach().float(), pos, cache, nq, nkv, hd)
    assert rel_err(out, ref) < 1e-2
    g = torch.randn_like(ref)
    out.backward(g.to(torch.bfloat16))
    gref = apply_rope_qkv_ref(g, pos, cache, nq, nkv, hd, inverse=True)
    assert rel_err(qkv.grad, gref) < 1e-2


def test_swiglu(cuda_device):
    from rl_b200.ops.activation import swiglu, swiglu_ref

    for F in (14336, 172):
        gu = torch.randn(33, 2 * F, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
        out = swiglu(gu)
        gr = gu.detach().float().requires_grad_(True)
        ref = swiglu_ref(gr)
        assert rel_err(out, ref) < 1e-2
        g = torch.randn_like(ref)
        out.backward(g.to(torch.bfloat16))
        ref.backward(g)
        assert rel_err(gu.grad, gr.grad) < 2e-2


def test_logprob_partials_and_grad(cuda_device):
    from rl_b200.ops.logprob import logits_entropy_ref, token_logprobs_and_entropy, token_logprobs_ref, \
        vocab_parallel_logprobs

    torch.manual_seed(1)
    for V in (128256, 1000):
        T = 40
        logits = (3 * torch.randn(T, V, device=cuda_device)).to(torch.bfloat16)
        tgt = torch.randint(0, V, (T,), device=cuda_device)
        for temp in (1.0, 0.7):
            lp, ent = token_logprobs_and_entropy(logits, tgt, temp)
            assert torch.allclose(lp, token_logprobs_ref(logits, tgt, temp), atol=2e-3, rtol=1e-3)
            assert torch.allclose(ent, logits_entropy_ref(logits, temp), atol=2e-3, rtol=1e-3)
        # gradient (in-place backward) vs autograd of the fp32 reference
        lg = logits.clone().requires_grad_(True)
        lp, _ = vocab_parallel_logprobs(lg, tgt, 0, 1.0, None, inplace_backward=False)
        g = torch.randn(T, device=cuda_device)
        lp.backward(g)
        lr = logits.float().requires_grad_(True)
        token_logprobs_ref(lr, tgt, 1.0).backward(g)
        assert rel_err(lg.grad, lr.grad) < 2e-2


def test_fused_linear_logprobs(cuda_device):
    from rl_b200.ops.fused_linear_logprob import linear_logprobs

    torch.manual_seed(2)
    T, H, V = 300, 256, 5000
    h = (torch.randn(T, H, device=cuda_device) * 0.5).to(torch.bfloat16).requires_grad_(True)
    W = (torch.randn(V, H, device=cuda_device) * 0.05).to(torch.bfloat16).requires_grad_(True)
    tgt = torch.randint(0, V, (T,), device=cuda_device)
    lp, ent = linear_logprobs(h, W, tgt, chunk=128)
    hr, Wr = h.detach().float().requires_grad_(True), W.detach().float().requires_grad_(True)
    lpr = torch.log_softmax(hr @ Wr.t(), -1).gather(-1, tgt[:, None]).squeeze(-1)
    assert torch.allclose(lp, lpr, atol=3e-2, rtol=1e-2)
    g = torch.randn(T, device=cuda_device)
    lp.backward(g)
    lpr.backward(g)
    assert rel_err(h.grad, hr.grad) < 3e-2
    assert rel_err(W.grad, Wr.grad) < 3e-2


def test_lm_head_logprob_epilogues(cuda_device):
    """The tcgen05 LM-head GEMM with the log-prob epilogues against an fp32
    PyTorch reference: softmax partials (logits never stored), entropy, target
    log-prob, vocabulary shards combined as under tensor parallelism, and the
    dlogits epilogue of the backward.  Shapes cover the 1-CTA and 2-CTA tiles,
    ragged row / vocabulary edges and targets outside a shard."""
    from rl_b200.ops._ext import ext
    from rl_b200.ops.logprob import _combine

    torch.manual_seed(5)
    for T, H, V, temp in ((300, 256, 5000, 1.0), (4096, 1024, 32000, 0.7), (77, 512, 1000, 1.3)):
        h = torch.randn(T, H, device=cuda_device).to(torch.bfloat16)
        W = (torch.randn(V, H, device=cuda_device) * (2.0 / H ** 0.5)).to(torch.bfloat16)
        tgt = torch.randint(0, V, (T,), device=cuda_device)
        x = (h.float() @ W.float().t()) / temp
        lse_r = torch.logsumexp(x, -1)
        lp_r = x.gather(1, tgt[:, None]).squeeze(1) - lse_r
        p_r = torch.softmax(x, -1)
        ent_r = lse_r - (p_r * x).sum(-1)
        m, s, u, xt = ext().gemm_logprob_partials(h, W, tgt.long(), float(temp))
        lse, lp, ent = _combine(m, s, u, xt, None)
        assert torch.allclose(lse, lse_r, atol=2e-3, rtol=1e-4), (T, V)
        assert torch.allclose(lp, lp_r, atol=2e-3, rtol=1e-4), (T, V)
        assert torch.allclose(ent, ent_r, atol=2e-3, rtol=1e-3), (T, V)
        # two vocabulary shards (the second not a multiple of 256 wide), combined by hand
        cut = (V // 2 // 8) * 8 + 8
        parts = []
        for lo, hi in ((0, cut), (cut, V)):
            parts.append(ext().gemm_logprob_partials(h, W[lo:hi].contiguous(), (tgt - lo).long(), float(temp)))
        gm = torch.maximum(parts[0][0], parts[1][0])
        ss = sum(pp[1] * torch.exp(pp[0] - gm) for pp in parts)
        lse2 = gm + torch.log(ss)
        lp2 = parts[0][3] + parts[1][3] - lse2
        assert torch.allclose(lp2, lp_r, atol=2e-3, rtol=1e-4), (T, V)
        # backward epilogue: dlogits = dlp / T * (onehot - softmax)
        dlp = torch.randn(T, device=cuda_device)
        d = ext().gemm_dlogits(h, W, tgt.long(), lse_r.contiguous(), dlp, float(temp))
        oh = torch.zeros_like(x).scatter_(1, tgt[:, None], 1.0)
        d_r = dlp[:, None] / temp * (oh - p_r)
        assert rel_err(d, d_r) < 1e-2, (T, V)


def test_sampling(cuda_device):
    from rl_b200.ops.sampling import sample_tokens

    torch.manual_seed(3)
    B, V = 8, 50000
    logits = torch.randn(B, V, device=cuda_device).to(torch.bfloat16)
    # top_k = 1 is greedy
    tok, lp = sample_tokens(logits, 1.0, top_k=1, top_p=1.0, seed=1)
    assert torch.equal(tok, logits.float().argmax(-1))
    assert torch.allclose(lp, torch.zeros_like(lp), atol=1e-5)
    # logprob of the sampled token under the full distribution
    tok, lp = sample_tokens(logits, 0.8, None, 1.0, seed=2)
    ref = torch.log_softmax(logits.float() / 0.8, -1).gather(-1, tok[:, None]).squeeze(-1)
    assert torch.allclose(lp, ref, atol=2e-3)
    # empirical distribution over a small vocabulary
    small = torch.tensor([[0.0, 1.0, 2.0, -1.0]], device=cuda_device).repeat(4096, 1)
    toks, _ = sample_tokens(small, 1.0, None, 1.0, seed=7)
    freq = torch.bincount(toks, minlength=4).float() / toks.numel()
    p = torch.softmax(small[0], -1)
    assert (freq - p).abs().max() < 0.03
    # top-p keeps the smallest prefix reaching the mass
    toks, lps = sample_tokens(small, 1.0, None, 0.8, seed=9)
    assert set(toks.unique().tolist()) <= {2, 1}
    kept = torch.softmax(torch.tensor([1.0, 2.0]), -1)
    assert torch.allclose(lps[toks == 2].mean().exp().cpu(), kept[1], atol=1e-3)
    # top-k = 2
    toks, _ = sample_tokens(small, 1.0, 2, 1.0, seed=11)
    assert set(toks.unique().tolist()) <= {1, 2}


def test_adamw(cuda_device):
    from rl_b200.ops.optim import adamw_step, adamw_step_ref, sum_of_squares

    n = 10007
    p = torch.randn(n, device=cuda_device)
    g = torch.randn(n, device=cuda_device)
    m = torch.zeros(n, device=cuda_device)
    v = torch.zeros(n, device=cuda_device)
    out = torch.empty(n, device=cuda_device, dtype=torch.bfloat16)
    p2, m2, v2 = p.clone(), m.clone(), v.clone()
    for step in (1, 2, 3):
        adamw_step(p, g, m, v, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, 0.5, out)
        adamw_step_ref(p2, g, m2, v2, 1e-3, 0.9, 0.999, 1e-8, 0.01, step, 0.5, None)
    assert torch.allclose(p, p2, atol=1e-6, rtol=1e-5)
    assert torch.allclose(out.float(), p2, atol=1e-2, rtol=1e-2)
    assert torch.allclose(sum_of_squares(g), g.pow(2).sum(), rtol=1e-4)


def test_fp8_quant(cuda_device):
    from rl_b200.ops.quant import dequant_fp8_block, quant_fp8_block, quant_fp8_block_ref, quant_fp8_group, \
        quant_fp8_group_ref

    w = torch.randn(300, 520, device=cuda_device).to(torch.bfloat16)
    for pow2 in (False, True):
        q, s = quant_fp8_block(w, 128, pow2)
        qr, sr = quant_fp8_block_ref(w, 128, pow2)
        assert torch.allclose(s, sr, rtol=1e-6)
        assert (q.float() - qr.float()).abs().max() <= 32.0  # at most one e4m3 ulp at the top of range
        assert rel_err(dequant_fp8_block(q, s), w.float()) < 0.05
    x = torch.randn(64, 512, device=cuda_device).to(torch.bfloat16)
    q, s = quant_fp8_group(x, 128, False)
    qr, sr = quant_fp8_group_ref(x, 128, False)
    assert torch.allclose(s, sr, rtol=1e-6)
    assert rel_err(q.float() * s.repeat_interleave(128, -1), x.float()) < 0.05


def _varlen(cuda_device, lens, nq, nkv, hd):
    T = sum(lens)
    qkv = torch.randn(T, (nq + 2 * nkv) * hd, device=cuda_device, dtype=torch.bfloat16)
    x = qkv.view(T, nq + 2 * nkv, hd)
    q, k, v = x[:, :nq], x[:, nq:nq + nkv], x[:, nq + nkv:]
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), device=cuda_device, dtype=torch.int32)
    return q, k, v, cu


@pytest.mark.parametrize("hd,nq,nkv", [(128, 8, 2), (64, 4, 4), (16, 4, 2)])
def test_flash_attention_fwd_bwd(cuda_device, hd, nq, nkv):
    from rl_b200.ops.attention import flash_attn_varlen, flash_attn_varlen_ref

    torch.manual_seed(4)
    lens = [1, 63, 64, 65, 200, 7]
    q, k, v, cu = _varlen(cuda_device, lens, nq, nkv, hd)
    q, k, v = (t.detach().requires_grad_(True) for t in (q, k, v))
    o = flash_attn_varlen(q, k, v, cu, max(lens), causal=True)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    oref, _ = flash_attn_varlen_ref(qr, kr, vr, cu, None, True)
    oref = oref.float()
    # recompute ref in fp32 with autograd
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    outs = []
    for b in range(len(lens)):
        s, e = int(cu[b]), int(cu[b + 1])
        qb = qf[s:e].transpose(0, 1)
        kb = kf[s:e].transpose(0, 1).repeat_interleave(nq // nkv, 0)
        vb = vf[s:e].transpose(0, 1).repeat_interleave(nq // nkv, 0)
        sc = (qb @ kb.transpose(-1, -2)) / math.sqrt(hd)
        sc = sc.masked_fill(torch.ones(e - s, e - s, device=cuda_device, dtype=torch.bool).triu(1), float("-inf"))
        outs.append((torch.softmax(sc, -1) @ vb).transpose(0, 1))
    of = torch.cat(outs)
    assert rel_err(o, of) < 2e-2
    g = torch.randn_like(of)
    o.backward(g.to(torch.bfloat16))
    of.backward(g)
    assert rel_err(q.grad, qf.grad) < 3e-2
    assert rel_err(k.grad, kf.grad) < 3e-2
    assert rel_err(v.grad, vf.grad) < 3e-2


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("nq,nkv", [(8, 2), (4, 4)])
def test_flash_attention_tcgen05_forward(cuda_device, causal, nq, nkv):
    """tcgen05 forward (csrc/attention_sm100.cu): output and log-sum-exp against an
    fp32 PyTorch reference on packed-QKV views, ragged lengths around the 128-query
    and 64-key tile edges."""
    ext = _ext.ext()
    torch.manual_seed(5)
    hd = 128
    lens = [1, 63, 64, 65, 127, 128, 129, 700, 2048, 33]
    q, k, v, cu = _varlen(cuda_device, lens, nq, nkv, hd)
    q = q * 2  # larger logits exercise the lazy rescaling
    q = q.to(torch.bfloat16)
    scale = hd ** -0.5
    qp = torch.empty(q.shape[0], nq + 2 * nkv, hd, device=cuda_device, dtype=torch.bfloat16)
    qp[:, :nq], qp[:, nq:nq + nkv], qp[:, nq + nkv:] = q, k, v
    q, k, v = qp[:, :nq], qp[:, nq:nq + nkv], qp[:, nq + nkv:]
    o, lse = ext.flash_attn_fwd_tc(q, k, v, cu, max(lens), scale, causal)
    torch.cuda.synchronize()
    assert ext.attn_tc_error_flag(True) == 0
    for b in range(len(lens)):
        s, e = int(cu[b]), int(cu[b + 1])
        qb = q[s:e].float().transpose(0, 1)
        kb = k[s:e].float().transpose(0, 1).repeat_interleave(nq // nkv, 0)
        vb = v[s:e].float().transpose(0, 1).repeat_interleave(nq // nkv, 0)
        sc = (qb @ kb.transpose(-1, -2)) * scale
        if causal:
            sc = sc.masked_fill(torch.ones(e - s, e - s, device=cuda_device, dtype=torch.bool).triu(1), float("-inf"))
        ref = (torch.softmax(sc, -1) @ vb).transpose(0, 1)
        assert rel_err(o[s:e], ref) < 1e-2, (b, lens[b])
        torch.testing.assert_close(lse[:, s:e], torch.logsumexp(sc, -1), atol=2e-2, rtol=1e-3)
    # same numbers as the mma.sync kernel it replaces
    o2, lse2 = ext.flash_attn_fwd(q, k, v, cu, max(lens), scale, causal)
    assert rel_err(o, o2) < 1e-2


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("nq,nkv", [(8, 2), (4, 4)])
def test_flash_attention_tcgen05_backward(cuda_device, causal, nq, nkv):
    """tcgen05 backward (csrc/attention_sm100.cu) against fp32 autograd on
    packed-QKV views: dq, dk, dv for ragged lengths around the 128-key tile and
    the 64-query block, GQA groups summed in-kernel."""
    ext = _ext.ext()
    torch.manual_seed(6)
    hd = 128
    lens = [1, 63, 64, 65, 127, 128, 129, 700, 1500, 33]
    q, k, v, cu = _varlen(cuda_device, lens, nq, nkv, hd)
    scale = hd ** -0.5
    o, lse = ext.flash_attn_fwd_tc(q, k, v, cu, max(lens), scale, causal)
    do = torch.randn_like(o)
    dq, dk, dv = ext.flash_attn_bwd_tc(do, q, k, v, o, lse, cu, max(lens), scale, causal)
    torch.cuda.synchronize()
    assert ext.attn_tc_error_flag(True) == 0
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    outs = []
    for b in range(len(lens)):
        s, e = int(cu[b]), int(cu[b + 1])
        qb = qf[s:e].transpose(0, 1)
        kb = kf[s:e].transpose(0, 1).repeat_interleave(nq // nkv, 0)
        vb = vf[s:e].transpose(0, 1).repeat_interleave(nq // nkv, 0)
        sc = (qb @ kb.transpose(-1, -2)) * scale
        if causal:
            sc = sc.masked_fill(torch.ones(e - s, e - s, device=cuda_device, dtype=torch.bool).triu(1), float("-inf"))
        outs.append((torch.softmax(sc, -1) @ vb).transpose(0, 1))
    of = torch.cat(outs)
    of.backward(do.float())
    assert rel_err(dq, qf.grad) < 3e-2, rel_err(dq, qf.grad)
    assert rel_err(dk, kf.grad) < 3e-2, rel_err(dk, kf.grad)
    assert rel_err(dv, vf.grad) < 3e-2, rel_err(dv, vf.grad)
    # and against the mma.sync backward it replaces
    dq2, dk2, dv2 = ext.flash_attn_bwd(do, q, k, v, o, lse, cu, max(lens), scale, causal)
    assert rel_err(dq, dq2) < 2e-2 and rel_err(dk, dk2) < 2e-2 and rel_err(dv, dv2) < 2e-2


@pytest.mark.parametrize("G,hd,bs", [(4, 128, 16), (8, 128, 16), (1, 128, 16), (4, 128, 256), (8, 64, 32),
                                     (2, 128, 8)])
def test_paged_decode_and_cache_write(cuda_device, G, hd, bs):
    from rl_b200.ops.attention import paged_decode_attention, paged_decode_attention_ref, write_kv_cache, \
        write_kv_cache_ref

    torch.manual_seed(5)
    B, nkv = 5, 4
    nq = nkv * G
    lens = torch.tensor([1, 17, 100, 600, 33], dtype=torch.int32)
    maxb = -(-1024 // bs)
    nblocks = B * maxb + 1
    kc = torch.zeros(nblocks, bs, nkv, hd, device=cuda_device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    bt = (torch.randperm(nblocks - 1)[: B * maxb].view(B, maxb) + 1).to(torch.int32).to(cuda_device)
    # fill the cache through the write kernel
    rows, slots = [], []
    for b in range(B):
        for t in range(int(lens[b])):
            slots.append(int(bt[b, t // bs]) * bs + t % bs)
    n = len(slots)
    kk = torch.randn(n, nkv, hd, device=cuda_device, dtype=torch.bfloat16)
    vv = torch.randn(n, nkv, hd, device=cuda_device, dtype=torch.bfloat16)
    sl = torch.tensor(slots, device=cuda_device)
    write_kv_cache(kk, vv, kc, vc, sl)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    write_kv_cache_ref(kk, vv, kc2, vc2, sl)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    q = torch.randn(B, nq, hd, device=cuda_device, dtype=torch.bfloat16)
    out = paged_decode_attention(q, kc, vc, bt, lens.to(cuda_device), max_seq_len=maxb * bs)
    ref = paged_decode_attention_ref(q, kc, vc, bt, lens, None)
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (1000, 6144, 4096), (384, 4096, 14336), (77, 128, 192),
                                   (4096, 768, 2048), (130, 96, 128)])
def test_gemm_tcgen05(cuda_device, M, N, K):
    ext = _ext.ext()
    torch.manual_seed(6)
    a = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    b = torch.randn(N, K, device=cuda_device).to(torch.bfloat16)
    c = ext.gemm_nt(a, b)
    torch.cuda.synchronize()
    assert ext.gemm_error_flag(True) == 0
    ref = a.float() @ b.float().t()
    assert rel_err(c, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (64, 4096, 4096), (64, 28672, 4096), (128, 4096, 14336),
                                   (200, 1000, 128), (33, 384, 4104), (256, 3072, 4096), (7, 128256, 512)])
def test_gemm_decode_tcgen05(cuda_device, M, N, K):
    ext = _ext.ext()
    torch.manual_seed(8)
    x = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    y = ext.gemm_decode(x, w)
    y2 = ext.gemm_decode(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    assert rel_err(y, ref) < 1e-2
    assert torch.equal(y, y2)  # split-K reduction is deterministic
    assert ext.gemm_decode_error_flag(True) == 0


@pytest.mark.parametrize("splits", [1, 2, 4, 8])
def test_gemm_decode_cluster_splits(cuda_device, splits):
    """Every K split (one CTA cluster per W tile, partials summed through
    distributed shared memory) gives the fp32 product, for 16..256 token rows."""
    ext = _ext.ext()
    torch.manual_seed(9)
    for M in (5, 32, 64, 100, 256):
        x = torch.randn(M, 2048, device=cuda_device).to(torch.bfloat16)
        w = (torch.randn(1280, 2048, device=cuda_device) * 0.05).to(torch.bfloat16)
        y = ext.gemm_decode_split(x, w, splits)
        torch.cuda.synchronize()
        assert rel_err(y, x.float() @ w.float().t()) < 1e-2, (M, splits)
    assert ext.gemm_decode_error_flag(True) == 0


@pytest.mark.parametrize("hd,G", [(128, 4), (64, 2)])
def test_flash_attn_segments_cp_layout(cuda_device, hd, G):
    """Context-parallel segment attention (query chunks vs key prefixes, shared
    keys) against the fp32 torch reference, forward and backward."""
    from rl_b200.ops.attention import flash_attn_segments
    from rl_b200.parallel.context_parallel import attention_segments_ref, cp_layout

    torch.manual_seed(9)
    lens = [300, 1000, 77]
    cp, nkv = 2, 2
    nq = nkv * G
    lay = cp_layout(lens, cp, 1, cuda_device, unit=16)
    Tq, Tk = lay.T_local, lay.T_full
    q = (torch.randn(Tq, nq, hd, device=cuda_device) * 0.5).to(torch.bfloat16).requires_grad_(True)
    k = (torch.randn(Tk, nkv, hd, device=cuda_device) * 0.5).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(Tk, nkv, hd, device=cuda_device).to(torch.bfloat16).requires_grad_(True)
    scale = hd ** -0.5
    o = flash_attn_segments(q, k, v, lay.q_start, lay.q_len, lay.k_start, lay.k_len, lay.max_q, lay.max_k, scale)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref = attention_segments_ref(qf, kf, vf, lay, scale)
    assert rel_err(o, ref) < 1e-2
    g = torch.randn_like(ref)
    o.backward(g.to(torch.bfloat16))
    ref.backward(g)
    assert rel_err(q.grad, qf.grad) < 3e-2
    assert rel_err(k.grad, kf.grad) < 3e-2
    assert rel_err(v.grad, vf.grad) < 3e-2


def _spec_case(B, V, k, device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    t_row = torch.randn(k + 1, V, generator=g) * 1.5
    d_row = torch.randn(k, V, generator=g) * 1.5
    tl = t_row.expand(B, k + 1, V).contiguous()
    dl = d_row.expand(B, k, V).contiguous()
    q = torch.softmax(d_row, -1)
    draft = torch.stack([torch.multinomial(q[i], B, replacement=True, generator=g) for i in range(k)], 1)
    return tl.to(device), dl.to(device), draft.to(device), torch.softmax(t_row, -1), q


def test_spec_verify_distribution_matches_target(cuda_device):
    """The first emitted token is distributed as the target's p_0 whatever the
    draft, and the acceptance rate of the first draft token is sum(min(p, q))."""
    from rl_b200.ops.spec_decode import spec_verify

    B, V, k = 60000, 6, 2
    tl, dl, draft, p, q = _spec_case(B, V, k, cuda_device)
    tok, n, lp = spec_verify(tl, dl, draft, temperature=1.0, seed=3)
    torch.cuda.synchronize()
    first = tok[:, 0].cpu()
    freq = torch.bincount(first, minlength=V).float() / B
    assert (freq - p[0]).abs().max() < 0.012, (freq, p[0])
    acc = (n.cpu() >= 2).float().mean()
    assert abs(float(acc) - float(torch.minimum(p[0], q[0]).sum())) < 0.012
    assert int(n.min()) >= 1 and int(n.max()) <= k + 1
    # logprobs are the target's log-probabilities of the emitted tokens
    lpt = torch.log(p[0])[first]
    assert torch.allclose(lp[:, 0].cpu(), lpt, atol=1e-4)
    # unused slots are -1
    idx = torch.arange(k + 1).unsqueeze(0)
    assert bool(((tok.cpu() == -1) == (idx >= n.cpu().unsqueeze(1))).all())


def test_spec_verify_greedy(cuda_device):
    from rl_b200.ops.spec_decode import spec_verify, spec_verify_ref

    B, V, k = 64, 1000, 2
    g = torch.Generator().manual_seed(4)
    tl = torch.randn(B, k + 1, V, generator=g)
    dl = torch.randn(B, k, V, generator=g)
    draft = tl[:, :k].argmax(-1)
    draft[::3, 0] = (draft[::3, 0] + 1) % V   # some first drafts wrong
    draft[1::3, 1] = (draft[1::3, 1] + 1) % V  # some second drafts wrong
    tok, n, lp = spec_verify(tl.to(cuda_device).to(torch.bfloat16), dl.to(cuda_device).to(torch.bfloat16),
                             draft.to(cuda_device), temperature=0.0)
    rt, rn, rlp = spec_verify_ref(tl.to(torch.bfloat16), dl.to(torch.bfloat16), draft, temperature=0.0)
    assert torch.equal(n.cpu(), rn) and torch.equal(tok.cpu(), rt)
    assert torch.allclose(lp.cpu(), rlp, atol=2e-2)


@pytest.mark.parametrize("M,N,K,splits", [(256, 512, 1024, 1), (1000, 6144, 4096, 0), (64, 4096, 4096, 0),
                                          (200, 320, 256, 1), (128, 128, 128, 0), (77, 1024, 2048, 3)])
def test_gemm_fp8_blockscaled(cuda_device, M, N, K, splits):
    """tcgen05 kind::f8f6f4 GEMM with per-128-K-block promotion against the fp32
    product of the same quantised operands (1x128 activation, 128x128 weight scales)."""
    from rl_b200.ops.fp8_gemm import gemm_fp8_ref
    from rl_b200.ops.quant import quant_fp8_block, quant_fp8_group

    ext = _ext.ext()
    torch.manual_seed(9)
    x = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    # weights with per-block magnitudes that differ, so wrong scale indexing shows
    w = torch.randn(N, K, device=cuda_device) * 0.05
    w = w * torch.rand(-(-N // 128), 1, -(-K // 128), 1, device=cuda_device).mul(4).add(0.25).expand(
        -1, 128, -1, 128).reshape(-(-N // 128) * 128, -(-K // 128) * 128)[:N, :K]
    w = w.to(torch.bfloat16)
    a_q, a_s = quant_fp8_group(x, 128, False)
    b_q, b_s = quant_fp8_block(w, 128, False)
    y = ext.gemm_fp8(a_q, a_s, b_q, b_s, splits)
    torch.cuda.synchronize()
    assert ext.gemm_fp8_error_flag(True) == 0
    ref = gemm_fp8_ref(a_q, a_s, b_q, b_s)
    assert rel_err(y, ref) < 5e-3
    # and close to the unquantised product (fp8 rounding only)
    assert rel_err(y, x.float() @ w.float().t()) < 6e-2


@pytest.mark.parametrize("M,N,K,splits", [(256, 448, 1024, 1), (1000, 6144, 4096, 0), (64, 4096, 4096, 0),
                                          (200, 320, 256, 1), (128, 224, 128, 1), (77, 1024, 2048, 3),
                                          (4096, 14336, 512, 1)])
def test_gemm_mxf8_hardware_block_scale(cuda_device, M, N, K, splits):
    """kind::mxf8f6f4.block_scale GEMM (power-of-two scales applied by the tensor
    cores from tensor memory) against the fp32 product of the same operands."""
    from rl_b200.ops.fp8_gemm import gemm_fp8_ref, mx_weight_scales, quant_act_mx
    from rl_b200.ops.quant import quant_fp8_block, quant_fp8_group

    ext = _ext.ext()
    torch.manual_seed(10)
    x = torch.randn(M, K, device=cuda_device).to(torch.bfloat16)
    w = torch.randn(N, K, device=cuda_device) * 0.05
    w = w * torch.rand(-(-N // 128), 1, -(-K // 128), 1, device=cuda_device).mul(16).add(0.1).expand(
        -1, 128, -1, 128).reshape(-(-N // 128) * 128, -(-K // 128) * 128)[:N, :K]
    w = w.to(torch.bfloat16)
    a_q, a_s = quant_fp8_group(x, 128, True)
    b_q, b_s = quant_fp8_block(w, 128, True)
    assert torch.equal(torch.exp2(torch.log2(b_s).round()), b_s)  # the quantiser's scales are powers of two
    a_q2, a_s_t = quant_act_mx(x)
    assert torch.equal(a_q2.view(torch.uint8), a_q.view(torch.uint8)) and torch.equal(a_s_t[:, :M], a_s.t())
    y = ext.gemm_mxf8(a_q, a_s_t, b_q, mx_weight_scales(b_s), splits)
    torch.cuda.synchronize()
    assert ext.gemm_fp8_error_flag(True) == 0
    ref = gemm_fp8_ref(a_q, a_s, b_q, b_s)
    assert rel_err(y, ref) < 5e-3


@pytest.mark.parametrize("counts,N,K", [([130, 0, 7, 300, 64], 256, 128), ([1, 1, 1, 1], 128, 64),
                                        ([513, 0, 0, 200], 384, 256), ([0, 0, 90], 1536, 512)])
def test_grouped_gemm_tcgen05(cuda_device, counts, N, K):
    """Per-expert tcgen05 GEMM (device-built tile schedule, tiles overhanging an
    expert's segment are not stored) against per-expert fp32 products."""
    ext = _ext.ext()
    torch.manual_seed(12)
    T, E = sum(counts), len(counts)
    x = torch.randn(T, K, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(E, N, K, device=cuda_device) * 0.05).to(torch.bfloat16)
    offs = torch.cumsum(torch.tensor(counts), 0).to(torch.int32).to(cuda_device)
    y = ext.grouped_gemm_nt(x, w, offs)
    torch.cuda.synchronize()
    assert ext.grouped_gemm_error_flag(True) == 0
    ref = torch.empty(T, N, device=cuda_device)
    s = 0
    for e, c in enumerate(counts):
        ref[s:s + c] = x[s:s + c].float() @ w[e].float().t()
        s += c
    assert rel_err(y, ref) < 1e-2


@pytest.mark.parametrize("T,E,k", [(1000, 128, 8), (37, 60, 4), (4096, 256, 8), (64, 1024, 1), (5, 8, 2)])
def test_moe_router_topk_kernel(T, E, k):
    """Router kernel vs the fp32 reference: probabilities, top-k ids, tokens per
    expert, the stable expert-grouped order, and the logits gradient of the
    renormalised top-k weights."""
    from rl_b200.ops.moe_router import router_topk, router_topk_ref

    torch.manual_seed(T + E)
    logits = (torch.randn(T, E, device="cuda") * 2).requires_grad_(True)
    probs, ids, counts, order = router_topk(logits, k)
    rp, rids, rcounts, _ = router_topk_ref(logits.detach(), k)
    torch.testing.assert_close(probs, rp, rtol=1e-5, atol=1e-6)
    # the chosen experts carry the k largest probabilities in descending order
    # (ids may differ from torch.topk only between probabilities within rounding)
    torch.testing.assert_close(rp.gather(-1, ids), rp.gather(-1, rids), rtol=1e-6, atol=1e-7)
    assert (ids == rids).float().mean() > 0.999
    assert torch.equal(counts.long(), torch.bincount(ids.reshape(-1), minlength=E))
    assert torch.equal(order, torch.argsort(ids.reshape(-1), stable=True))
    w = probs.gather(-1, ids)
    (w / w.sum(-1, keepdim=True) * torch.arange(1, k + 1, device="cuda")).sum().backward()
    g = logits.grad.clone()
    lr = logits.detach().clone().requires_grad_(True)
    p2 = torch.softmax(lr, -1)
    w2 = p2.gather(-1, ids)
    (w2 / w2.sum(-1, keepdim=True) * torch.arange(1, k + 1, device="cuda")).sum().backward()
    torch.testing.assert_close(g, lr.grad, rtol=1e-4, atol=1e-6)
