"""Kernel micro-benchmarks (CUDA-event timing, warm-up first) for the native kernels.

    python -m rl_b200.bench_kernels gemm      [M N K]
    python -m rl_b200.bench_kernels decode    [B L]
    python -m rl_b200.bench_kernels decode_gemm [M]
    python -m rl_b200.bench_kernels attn      [T_per_seq n_seq]
    python -m rl_b200.bench_kernels logprob   [T V]
    python -m rl_b200.bench_kernels lmhead    [T H V]
    python -m rl_b200.bench_kernels lmhead_fwd [T H V]   (fused forward only: the ncu case)
    python -m rl_b200.bench_kernels fp8       [M N K]
    python -m rl_b200.bench_kernels numerics  [prompts max_new]
    python -m rl_b200.bench_kernels rollout   [seqs max_new]   (8B rollout; NVTX range "rollout_timed")

Each prints one line with the time and the achieved rate, and is small enough
to be captured under ``ncu -k <kernel> -c 1`` (a few GB on the device at most).
"""

from __future__ import annotations

import sys

import torch


def _time(fn, reps: int = 10, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps  # ms


def bench_gemm(M=8192, N=8192, K=4096):
    """The three products of a linear layer on the tcgen05 kernel (1-CTA 128x256 and
    2-CTA 256x256 tiles) against the library GEMM on the same operands."""
    from rl_b200.ops._ext import ext

    dev = torch.device("cuda")
    C = ext()
    fl = 2 * M * N * K
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)      # [M, K]
    xt = torch.randn(K, M, device=dev).to(torch.bfloat16)     # [K, M]
    w = torch.randn(N, K, device=dev).to(torch.bfloat16)      # [N, K]
    wt = torch.randn(K, N, device=dev).to(torch.bfloat16)     # [K, N]
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    acc = torch.zeros(M, N, device=dev, dtype=torch.float32)
    cases = [
        ("nt (fprop)", x, w, False, False, out, False, lambda: torch.matmul(x, w.t())),
        ("nn (dgrad)", x, wt, False, True, out, False, lambda: torch.matmul(x, wt)),
        ("tn (wgrad)", xt, wt, True, True, out, False, lambda: torch.matmul(xt.t(), wt)),
        ("tn += fp32", xt, wt, True, True, acc, True, lambda: acc.add_(torch.mm(xt.t(), wt, out_dtype=torch.float32))),
    ]
    for name, a, b, amn, bmn, o, add, lib in cases:
        res = []
        for tile in (1, 2):
            t = _time(lambda: C.gemm_sm100(a, b, o, amn, bmn, add, tile))
            res.append(f"{'1cta' if tile == 1 else '2cta'} {t:.3f} ms {fl / t / 1e9:.1f}")
        tl = _time(lib)
        print(f"gemm {name} {M}x{N}x{K}: " + " | ".join(res) + f" | library {tl:.3f} ms {fl / tl / 1e9:.1f} TFLOP/s")
    assert C.gemm_sm100_error_flag(True) == 0


def bench_decode(B=64, L=1024, nkv=8, G=4, hd=128, bs=256):
    from rl_b200.ops.attention import paged_decode_attention

    dev = torch.device("cuda")
    per = L // bs + 1
    kc = torch.randn(B * per + 1, bs, nkv, hd, device=dev).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = (torch.arange(B * per).view(B, per) + 1).to(torch.int32).to(dev)
    sl = torch.full((B,), L, dtype=torch.int32, device=dev)
    q = torch.randn(B, nkv * G, hd, device=dev).to(torch.bfloat16)
    t = _time(lambda: paged_decode_attention(q, kc, vc, bt, sl, max_seq_len=per * bs), reps=20)
    byts = B * L * nkv * hd * 2 * 2
    print(f"paged_decode B={B} L={L}: {t * 1e3:.1f} us {byts / (t * 1e-3) / 1e12:.2f} TB/s")


def bench_router(T=16384, E=128, k=8):
    """MoE router kernel (softmax, top-k, counts, stable expert-grouped order)
    against the PyTorch ops it replaces (softmax, topk, bincount, stable argsort)."""
    from rl_b200.ops.moe_router import router_topk, router_topk_ref

    logits = torch.randn(T, E, device="cuda")
    t_n = _time(lambda: router_topk(logits, k), reps=50)
    t_r = _time(lambda: router_topk_ref(logits, k), reps=50)
    byts = T * E * 4 * 2 + T * k * 8 * 3  # logits read + probs written, ids / order / pos
    print(f"router T={T} E={E} k={k}: native {t_n * 1e3:.1f} us ({byts / (t_n * 1e-3) / 1e9:.0f} GB/s), "
          f"torch {t_r * 1e3:.1f} us, speed-up {t_r / t_n:.2f}x")


def bench_decode_gemm(M=64):
    """The Llama-3.1-8B linear layers at decode batch M (weight-streaming bound):
    time and achieved weight bandwidth per projection.  Each timed call reads a
    different copy of the weight (copies > 2x L2 in total), as consecutive
    layers of a decode step do, so no weight is served from L2."""
    dev = torch.device("cuda")
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336),
              "lm_head": (128256, 4096)}
    from rl_b200.ops._ext import ext

    tp = int(__import__("os").environ.get("RLB_BENCH_TP", "1"))
    tot_t, tot_l, tot_b = 0.0, 0.0, 0
    for name, (N, K) in shapes.items():
        if tp > 1:  # this rank's shard: column-parallel split N, row-parallel split K
            N, K = (N, K // tp) if name in ("o", "down") else (N // tp, K)
        byts = N * K * 2
        copies = max(2, -(-300 * 2 ** 20 // byts))
        ws = [torch.randn(N, K, device=dev).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        i = [0]

        def nxt():
            i[0] = (i[0] + 1) % copies
            return ws[i[0]]

        reps = max(20, copies)
        t = _time(lambda: ext().gemm_decode(x, nxt()), reps=reps)
        tl = _time(lambda: torch.matmul(x, nxt().t()), reps=reps)
        del ws
        mult = 32 if name != "lm_head" else 1
        tot_t += t * mult
        tot_l += tl * mult
        tot_b += byts * mult
        print(f"decode gemm {name} M={M} N={N} K={K}: native {t * 1e3:.1f} us {byts / (t * 1e-3) / 1e12:.2f} TB/s | "
              f"library {tl * 1e3:.1f} us {byts / (tl * 1e-3) / 1e12:.2f} TB/s")
    print(f"decode gemms per token step (32 layers + head, tp={tp}): native {tot_t:.3f} ms "
          f"{tot_b / (tot_t * 1e-3) / 1e12:.2f} TB/s | library {tot_l:.3f} ms {tot_b / (tot_l * 1e-3) / 1e12:.2f} TB/s")
    assert ext().gemm_decode_error_flag(True) == 0


def bench_attn(L=2048, n=8, nq=32, nkv=8, hd=128):
    """Causal varlen attention (n sequences of L tokens, GQA nq:nkv): the tcgen05
    forward, the mma.sync forward and backward, and torch SDPA (cuDNN backend)."""
    from rl_b200.ops._ext import ext
    from rl_b200.ops.attention import flash_attn_varlen

    dev = torch.device("cuda")
    T = L * n
    q = torch.randn(T, nq, hd, device=dev).to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(T, nkv, hd, device=dev).to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(T, nkv, hd, device=dev).to(torch.bfloat16).requires_grad_(True)
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
    sc = hd ** -0.5
    fl = 4 * n * L * L / 2 * hd * nq
    C = ext()
    res = []
    if hd == 128:
        t = _time(lambda: C.flash_attn_fwd_tc(q.detach(), k.detach(), v.detach(), cu, L, sc, True))
        res.append(f"fwd tcgen05 {t:.3f} ms {fl / t / 1e9:.1f}")
    t = _time(lambda: C.flash_attn_fwd(q.detach(), k.detach(), v.detach(), cu, L, sc, True))
    res.append(f"fwd mma.sync {t:.3f} ms {fl / t / 1e9:.1f}")
    o, lse = C.flash_attn_fwd(q.detach(), k.detach(), v.detach(), cu, L, sc, True)
    g = torch.randn_like(o)
    if hd == 128:
        tb = _time(lambda: C.flash_attn_bwd_tc(g, q.detach(), k.detach(), v.detach(), o, lse, cu, L, sc, True))
        res.append(f"bwd tcgen05 {tb:.3f} ms {2.5 * fl / tb / 1e9:.1f}")
    tb = _time(lambda: C.flash_attn_bwd(g, q.detach(), k.detach(), v.detach(), o, lse, cu, L, sc, True))
    res.append(f"bwd mma.sync {tb:.3f} ms {2.5 * fl / tb / 1e9:.1f}")
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel

        qb = q.detach().view(n, L, nq, hd).transpose(1, 2).contiguous().requires_grad_(True)
        kb = k.detach().view(n, L, nkv, hd).transpose(1, 2).repeat_interleave(nq // nkv, 1).contiguous() \
            .requires_grad_(True)
        vb = v.detach().view(n, L, nkv, hd).transpose(1, 2).repeat_interleave(nq // nkv, 1).contiguous() \
            .requires_grad_(True)
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            f = lambda: torch.nn.functional.scaled_dot_product_attention(qb, kb, vb, is_causal=True)  # noqa: E731
            ts = _time(f)
            ob = f()
            gb = torch.randn_like(ob)
            tsb = _time(lambda: torch.autograd.grad(ob, (qb, kb, vb), gb, retain_graph=True))
        res.append(f"cuDNN SDPA fwd {ts:.3f} ms {fl / ts / 1e9:.1f} bwd {tsb:.3f} ms {2.5 * fl / tsb / 1e9:.1f}")
    except Exception as e:  # noqa: BLE001
        res.append(f"cuDNN SDPA unavailable ({type(e).__name__})")
    print(f"flash_attn L={L} n={n} nq={nq} nkv={nkv}: " + " | ".join(res) + " TFLOP/s")
    if hd == 128:
        assert C.attn_tc_error_flag(True) == 0


def bench_fp8(M=8192, N=8192, K=8192):
    """Block-scaled e4m3 GEMM (activation quantisation excluded) against the
    library bf16 GEMM and the library fp8 GEMM with one scale per tensor."""
    from rl_b200.ops._ext import ext
    from rl_b200.ops.quant import quant_fp8_block, quant_fp8_group

    dev = torch.device("cuda")
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev) * 0.05).to(torch.bfloat16)
    a_q, a_s = quant_fp8_group(x, 128, False)
    b_q, b_s = quant_fp8_block(w, 128, False)
    t = _time(lambda: ext().gemm_fp8(a_q, a_s, b_q, b_s, 0))
    from rl_b200.ops.fp8_gemm import mx_weight_scales, quant_act_mx

    p_q, p_s = quant_act_mx(x)
    w_q, w_s = quant_fp8_block(w, 128, True)
    w_st = mx_weight_scales(w_s)
    tm = _time(lambda: ext().gemm_mxf8(p_q, p_s, w_q, w_st, 0))
    tmq = _time(lambda: quant_act_mx(x))
    tq = _time(lambda: quant_fp8_group(x, 128, False))
    tl = _time(lambda: torch.matmul(x, w.t()))
    one = torch.ones((), device=dev)
    try:
        ts = _time(lambda: torch._scaled_mm(a_q, b_q.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16))
        lib8 = f" | library fp8 per-tensor {ts:.3f} ms {2 * M * N * K / ts / 1e9:.1f} TFLOP/s"
    except Exception as e:  # noqa: BLE001 - report what the library does not support
        lib8 = f" | library fp8 unavailable ({type(e).__name__})"
    fl = 2 * M * N * K
    byts = M * K + N * K + M * N * 2
    print(f"gemm_mxf8 {M}x{N}x{K}: {tm:.3f} ms {fl / tm / 1e9:.1f} TFLOP/s {byts / (tm * 1e-3) / 1e12:.2f} TB/s "
          f"(+ act quant {tmq:.3f} ms)")
    print(f"gemm_fp8 {M}x{N}x{K}: {t:.3f} ms {fl / t / 1e9:.1f} TFLOP/s {byts / (t * 1e-3) / 1e12:.2f} TB/s "
          f"(+ act quant {tq:.3f} ms) | library bf16 {tl:.3f} ms {fl / tl / 1e9:.1f} TFLOP/s{lib8}")


def bench_logprob(T=8192, V=128256):
    from rl_b200.ops.logprob import token_logprobs_and_entropy

    dev = torch.device("cuda")
    x = torch.randn(T, V, device=dev).to(torch.bfloat16)
    tg = torch.randint(0, V, (T,), device=dev)
    t = _time(lambda: token_logprobs_and_entropy(x, tg))
    print(f"logprob T={T} V={V}: {t:.3f} ms {T * V * 2 / (t * 1e-3) / 1e12:.2f} TB/s")


def bench_lmhead(T=8192, H=4096, V=128256):
    """LM head + log-prob / entropy, forward and backward, on the fused tcgen05
    epilogues against the two-pass path (logits tile stored as bf16, then a
    separate reduction / gradient kernel), same GEMM kernels otherwise."""
    from rl_b200.ops import gemm as G
    from rl_b200.ops._ext import ext
    from rl_b200.ops.logprob import _bwd_inplace, _combine, logprob_partials

    dev = torch.device("cuda")
    C = ext()
    h = torch.randn(T, H, device=dev).to(torch.bfloat16)
    W = (torch.randn(V, H, device=dev) * H ** -0.5).to(torch.bfloat16)
    tg = torch.randint(0, V, (T,), device=dev)
    dlp = torch.randn(T, device=dev)
    acc = torch.zeros(V, H, device=dev)
    fl = 2 * T * H * V

    def fwd_fused():
        return _combine(*C.gemm_logprob_partials(h, W, tg, 1.0), None)

    def fwd_two_pass():
        lg = G.mm_nt(h, W)
        return _combine(*logprob_partials(lg, tg, 1.0), None)

    lse = fwd_fused()[0]

    def bwd_fused():
        d = C.gemm_dlogits(h, W, tg, lse, dlp, 1.0)
        G.mm_nn(d, W)
        G.mm_tn_accumulate(d, h, acc)

    def bwd_two_pass():
        lg = G.mm_nt(h, W)
        _bwd_inplace(dlp, lg, tg, lse, 1.0, lg)
        G.mm_nn(lg, W)
        G.mm_tn_accumulate(lg, h, acc)

    tf, t2 = _time(fwd_fused), _time(fwd_two_pass)
    tb, tb2 = _time(bwd_fused), _time(bwd_two_pass)
    tg_ = _time(lambda: G.mm_nt(h, W))
    wb = (V * H + T * H) * 2
    print(f"lmhead fwd T={T} H={H} V={V}: fused {tf:.3f} ms {fl / tf / 1e9:.1f} TFLOP/s | two-pass {t2:.3f} ms | "
          f"GEMM alone (bf16 logits out) {tg_:.3f} ms | weight+hidden bytes / fused time "
          f"{wb / (tf * 1e-3) / 1e12:.2f} TB/s")
    print(f"lmhead bwd: fused {tb:.3f} ms {3 * fl / tb / 1e9:.1f} TFLOP/s | two-pass {tb2:.3f} ms")


def bench_lmhead_fwd(T=4096, H=4096, V=128256):
    """Only the fused LM-head log-prob forward (GEMM + tile merge), 3 warm-up and
    10 timed launches: the small case for an ncu capture of its GEMM."""
    from rl_b200.ops._ext import ext

    dev = torch.device("cuda")
    h = torch.randn(T, H, device=dev).to(torch.bfloat16)
    W = (torch.randn(V, H, device=dev) * H ** -0.5).to(torch.bfloat16)
    tg = torch.randint(0, V, (T,), device=dev)
    t = _time(lambda: ext().gemm_logprob_partials(h, W, tg, 1.0))
    fl = 2 * T * H * V
    print(f"lmhead_fwd T={T} H={H} V={V}: {t:.3f} ms {fl / t / 1e9:.1f} TFLOP/s")


def bench_numerics(prompts=64, max_new=256):
    """Rollout-vs-trainer log-prob agreement on the Llama-3.1-8B shape (random
    init): ``gen_kl_error`` (k3 estimator, as GRPO reports it) between the rollout
    engine's sampled-token log-probs and the trainer's, and, as the floor it can
    be read against, the same statistic between two trainer forwards that differ
    only in the attention kernel (tcgen05 vs mma.sync).  A random 32-layer model
    amplifies last-bit differences of any two valid kernels into log-prob noise;
    this measures how much."""
    import json
    import math

    import rl_b200.ops.attention as attn
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import single_process_state

    dev = torch.device("cuda", 0)
    mcfg = get_model_config("llama3.1-8b")
    pcfg = {"model_name": "llama3.1-8b", "max_total_sequence_length": 512 + max_new, "precision": "bfloat16",
            "train_global_batch_size": prompts,
            "generation": {"temperature": 1.0, "top_p": 1.0, "top_k": None, "max_new_tokens": max_new,
                           "max_num_seqs": 512, "mcore_generation_config": {"block_size_tokens": 256}},
            "sequence_packing": {"train_mb_tokens": 16384, "logprob_mb_tokens": 32768}}
    w = PolicyWorker(pcfg, model_cfg=mcfg, pstate=single_process_state(dev), seed=1234)
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(128, 513, (prompts,), generator=g)
    ids = torch.randint(0, mcfg.vocab_size, (prompts, 512), generator=g)
    out = w.generate(BatchedDataDict({"input_ids": ids, "input_lengths": lens}))
    S = out["output_ids"].shape[1]
    mask = torch.zeros(prompts, S, dtype=torch.bool)
    for r in range(prompts):
        mask[r, int(lens[r]):int(out["unpadded_sequence_lengths"][r])] = True
    seqs = BatchedDataDict({"input_ids": out["output_ids"], "input_lengths": out["unpadded_sequence_lengths"]})

    def k3(a, b):
        d = (a.float() - b.float())[mask]
        return float((torch.exp(d) - d - 1).mean()), float(d.pow(2).mean().sqrt())

    lp = w.get_logprobs(seqs)["logprobs"]
    gen_kl, gen_rms = k3(lp, out["logprobs"])
    attn._ATTN_TC = not attn._ATTN_TC
    try:
        lp2 = w.get_logprobs(seqs)["logprobs"]
    finally:
        attn._ATTN_TC = not attn._ATTN_TC
    self_kl, self_rms = k3(lp2, lp)
    print(json.dumps({"gen_kl_error": gen_kl, "gen_rms_dlogp": gen_rms, "trainer_vs_trainer_other_attention_kl": self_kl,
                      "trainer_vs_trainer_rms_dlogp": self_rms, "tokens": int(mask.sum()),
                      "threshold": 0.002, "ln_vocab": math.log(mcfg.vocab_size)}))


def bench_rollout(seqs=64, max_new=256):
    """Rollout engine on the Llama-3.1-8B shape (random init): one warm-up
    generate (captures the decode graphs), then one timed generate inside the
    NVTX range ``rollout_timed`` (``ncu --nvtx --nvtx-include rollout_timed/``
    restricts a launch list to it).  Prompts U[128, 512], EOS ignored."""
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import single_process_state

    dev = torch.device("cuda", 0)
    mcfg = get_model_config("llama3.1-8b")
    pcfg = {"model_name": "llama3.1-8b", "max_total_sequence_length": 512 + max_new, "precision": "bfloat16",
            "train_global_batch_size": seqs,
            "generation": {"temperature": 1.0, "top_p": 1.0, "top_k": None, "max_new_tokens": max_new,
                           "max_num_seqs": 512, "mcore_generation_config": {"block_size_tokens": 256}}}
    w = PolicyWorker(pcfg, model_cfg=mcfg, pstate=single_process_state(dev), seed=1234, init_reference_model=False)
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(128, 513, (seqs,), generator=g)
    ids = torch.randint(0, mcfg.vocab_size, (seqs, 512), generator=g)
    batch = BatchedDataDict({"input_ids": ids, "input_lengths": lens})
    w.generate(batch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("rollout_timed")
    e0.record()
    out = w.generate(batch)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1)
    n = int(out["generation_lengths"].sum())
    print(f"rollout seqs={seqs} max_new={max_new}: {t:.1f} ms, {n / t * 1e3:.0f} generated tok/s, "
          f"{t / max_new:.3f} ms per decode step (incl. prefill share)")


def bench_longctx(seq=32768, steps=2):
    """Long-context training on one GPU: the Llama-3.1-8B shape (random init),
    one packed sequence of ``seq`` tokens per step (activation checkpointing,
    GRPO clipped-PG loss, optimizer step), timed with CUDA events after a warm-up
    step; prints step time, tokens/s, model TFLOP/s and peak memory."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import single_process_state
    from rl_b200.utils.flops import forward_flops

    dev = torch.device("cuda", 0)
    mcfg = get_model_config("llama3.1-8b")
    pcfg = {"model_name": "llama3.1-8b", "max_total_sequence_length": seq, "precision": "bfloat16",
            "train_global_batch_size": 1, "max_grad_norm": 1.0,
            "optimizer": {"kwargs": {"lr": 1e-7, "weight_decay": 0.0}},
            "megatron_cfg": {"activation_checkpointing": True},
            "generation": {"max_new_tokens": 8, "mcore_generation_config": {"block_size_tokens": 256}},
            "sequence_packing": {"train_mb_tokens": seq, "logprob_mb_tokens": seq}}
    w = PolicyWorker(pcfg, model_cfg=mcfg, pstate=single_process_state(dev), seed=1234, init_reference_model=False)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, mcfg.vocab_size, (1, seq), generator=g)
    tm = torch.zeros(1, seq)
    tm[0, seq // 8:] = 1.0
    lp = -torch.rand(1, seq, generator=g) * tm
    data = BatchedDataDict({"input_ids": ids, "input_lengths": torch.tensor([seq]), "advantages": tm * 0.5,
                            "generation_logprobs": lp, "prev_logprobs": lp.clone(), "token_mask": tm,
                            "sample_mask": torch.ones(1)})
    # rollout-consistent log-probs (ratio 1 at the first step), so the update is a real one
    cur = w.get_logprobs(data)["logprobs"].float().cpu() * tm
    data["generation_logprobs"], data["prev_logprobs"] = cur, cur.clone()
    lf = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    w.train(data, lf)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        res = w.train(data, lf)
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / steps / 1e3
    fl = 3.0 * forward_flops(mcfg, [seq])  # forward + backward
    print(f"longctx seq={seq}: {t * 1e3:.0f} ms per step, {seq / t:.0f} tokens/s, "
          f"{fl / t / 1e12:.0f} model TFLOP/s (fwd+bwd, recompute excluded), "
          f"peak {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB, loss {res['loss']:.4f}, "
          f"grad_norm {res['grad_norm']:.3f}")


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    what = argv.pop(0) if argv else "gemm"
    args = [int(x) for x in argv]
    torch.manual_seed(0)
    {"gemm": bench_gemm, "decode": bench_decode, "decode_gemm": bench_decode_gemm, "attn": bench_attn,
     "logprob": bench_logprob, "lmhead": bench_lmhead, "lmhead_fwd": bench_lmhead_fwd, "fp8": bench_fp8, "numerics": bench_numerics,
     "rollout": bench_rollout, "longctx": bench_longctx, "router": bench_router}[what](*args)


if __name__ == "__main__":
    main()
