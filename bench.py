#!/usr/bin/env python
"""GRPO step benchmark on the Llama-3.1-8B shape (the reference's headline GRPO metric).

Config: Llama-3.1-8B architecture (32 layers, hidden 4096,
32 / 8 heads, head dim 128, SwiGLU 14336, vocab 128256, RoPE theta 5e5), random
init, bf16, colocated rollout + train with the full refit every step; 8 samples
per prompt, prompt lengths uniform in [128, 512] with tokens uniform over the
vocabulary, max 1024 new tokens, deterministic seeded-hash reward.  Weak scaling:
8 prompts (64 samples) per GPU; TP=2 when N >= 2 (TP2 x DP(N/2)), TP=1 on one GPU.

Timing: W untimed warm-up GRPO steps, then K timed steps bracketed by a barrier
and a device synchronize; device time from CUDA events on the launching stream,
max over ranks.  ``value`` is the whole-job rollout+train tokens/s (prompt +
generated tokens of all samples / step time).  ``e2e`` is the same metric by
host wall clock through the public API (``grpo_train``), including the pinned
host->device copy of every step's prompts and the device->host read of the loss.

``--impl reference`` runs the unmodified reference from ``baseline/_ref`` when it
is importable, otherwise prints its ``unavailable`` line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# one big model state + a KV cache that is freed and re-created every step: let the
# caching allocator grow segments instead of fragmenting HBM
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

METRIC = "GRPO step time & rollout+train tokens/s (8×B200, max over ranks) at 8B"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--model", default="llama3.1-8b")
    p.add_argument("--prompts-per-gpu", type=int, default=8)
    p.add_argument("--generations", type=int, default=8)
    p.add_argument("--min-prompt", type=int, default=128)
    p.add_argument("--max-prompt", type=int, default=512)
    p.add_argument("--max-new", type=int, default=1024)
    p.add_argument("--tp", type=int, default=0, help="0 = 2 when gpus >= 2 else 1")
    p.add_argument("--sp", type=int, default=-1,
                   help="sequence parallelism (fused GEMM + reduce-scatter kernels) under TP; -1 = on when tp > 1")
    p.add_argument("--gen-tp", type=int, default=0,
                   help="rollout tensor parallelism: 0 = training TP (in-place refit), 1 = full rollout weights per GPU "
                        "(refit reshards over NVLink)")
    p.add_argument("--act-ckpt", type=int, default=-1,
                   help="activation checkpointing: -1 = on for one GPU (memory), off when TP >= 2 (activations fit)")
    p.add_argument("--mb-tokens", type=int, default=16384)
    p.add_argument("--kl", type=float, default=0.01)
    p.add_argument("--layers", type=int, default=0, help="debug only: override layer count (invalid for scoring)")
    p.add_argument("--preset", default="llama8b", choices=sorted(PRESETS),
                   help="llama8b: the headline config (BASELINE config 2); qwen30b_a3b_ep8: config 3 "
                        "(MoE, EP over all GPUs); qwen32b_fp8_tp4: config 5 (block-scaled fp8 training and "
                        "rollout, fp8 KV cache, 2-token draft)")
    args = p.parse_args()
    pre = PRESETS[args.preset]
    for k, v in pre.get("args", {}).items():  # a preset fills the arguments left at their defaults
        if getattr(args, k) == p.get_default(k):
            setattr(args, k, v)
    return args


# Per-GPU work of the reference's benchmark configs (weak scaling: prompts scale with N).
PRESETS = {
    "llama8b": {"model_label": "Llama-3.1-8B-shape", "args": {}},
    "qwen30b_a3b_ep8": {"model_label": "Qwen3-30B-A3B-shape", "ep": "all", "tp": 1,
                        "args": {"model": "qwen3-30b-a3b", "prompts_per_gpu": 4, "generations": 16,
                                 "min_prompt": 256, "max_prompt": 256, "max_new": 2048, "act_ckpt": 1}},
    "qwen32b_fp8_tp4": {"model_label": "Qwen3-32B-shape fp8", "tp": 4, "fp8": True,
                        "args": {"model": "qwen3-32b", "prompts_per_gpu": 4, "generations": 8,
                                 "min_prompt": 512, "max_prompt": 512, "max_new": 4096, "act_ckpt": 1}},
}


def reference_arm(args) -> None:
    """Run the unmodified reference from ``baseline/_ref`` through its public GRPO entry
    point when it imports; otherwise print why it cannot run, as one ``unavailable`` line."""
    why = None
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "nemo_rl")):
        why = "reference not installed under baseline/_ref (the folder holds no nemo_rl package)"
    else:
        sys.path.insert(0, ref)
        missing = []
        for mod in ("ray", "megatron.core", "vllm"):
            try:
                __import__(mod)
            except Exception as e:  # noqa: BLE001
                missing.append(f"{mod} ({type(e).__name__})")
        try:
            import nemo_rl.algorithms.grpo  # noqa: F401
        except Exception as e:  # noqa: BLE001
            why = (f"reference GRPO not importable from baseline/_ref ({type(e).__name__}: {e}); the offline "
                   f"install carries only the top-level nemo_rl package, and its GRPO driver also needs "
                   f"{', '.join(missing) or 'its Ray worker groups'}, which are not in this image or wheelhouse")
        if why is None and missing:
            why = f"reference GRPO imported but its Ray-based driver cannot start: missing {', '.join(missing)}"
    if why is None:
        why = "reference imported but no GPU launcher for its Ray single controller exists in this image"
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def reader():
            for line in self.proc.stdout:
                self.rows.append([x.strip() for x in line.split(",")])

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    from rl_b200.algorithms.grpo import GRPOSaveState, grpo_train
    from rl_b200.data.datasets import StatefulDataLoader, SyntheticPromptDataset
    from rl_b200.environments.synthetic import HashRewardEnvironment
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.ops import _ext
    from rl_b200.parallel.state import init_distributed
    from rl_b200.utils.timer import max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    pre = PRESETS[args.preset]
    tp = args.tp or pre.get("tp") or (2 if args.gpus >= 2 else 1)
    tp = min(tp, args.gpus)
    ep = args.gpus // tp if pre.get("ep") == "all" else 1
    ps = init_distributed(tp=tp, ep=ep, timeout_s=900)
    dev = ps.device
    if not _ext.has_ext():
        raise SystemExit(f"native extension not loaded: {_ext._ERR!r}")
    mcfg = get_model_config(args.model)
    if args.layers:
        mcfg = mcfg.replace(num_layers=args.layers)
    max_len = args.max_prompt + args.max_new
    prompts_global = args.prompts_per_gpu * args.gpus
    G = args.generations
    pcfg = {
        "model_name": args.model, "max_total_sequence_length": max_len, "precision": "bfloat16",
        "train_global_batch_size": prompts_global * G, "train_micro_batch_size": 8,
        "logprob_chunk_size": 4096, "max_grad_norm": 1.0,
        "optimizer": {"name": "torch.optim.AdamW",
                      "kwargs": {"lr": 3e-7, "weight_decay": 0.01, "betas": [0.9, 0.999], "eps": 1e-8}},
        "megatron_cfg": {"activation_checkpointing": (tp < 2) if args.act_ckpt < 0 else bool(args.act_ckpt),
                         "sequence_parallel": (tp > 1) if args.sp < 0 else bool(args.sp),
                         "expert_model_parallel_size": ep,
                         **({"fp8_cfg": {"enabled": True, "fp8": "e4m3", "fp8_recipe": "blockwise"}}
                            if pre.get("fp8") else {})},
        "generation": {"temperature": 1.0, "top_p": 1.0, "top_k": None, "max_new_tokens": args.max_new,
                       "max_num_seqs": 512, "mcore_generation_config": {"block_size_tokens": 256},
                       "tensor_parallel_size": args.gen_tp or tp,
                       **({"vllm_cfg": {"precision": "fp8", "kv_cache_dtype": "fp8"},
                           "speculative": {"num_speculative_tokens": 2, "draft_num_layers": 1}}
                          if pre.get("fp8") else {})},
        "sequence_packing": {"train_mb_tokens": args.mb_tokens, "logprob_mb_tokens": args.mb_tokens * 2},
    }
    cfg = {
        "grpo": {"num_prompts_per_step": prompts_global, "num_generations_per_prompt": G,
                 "max_num_steps": args.warmup + args.steps, "seed": 42},
        "loss_fn": {"reference_policy_kl_penalty": args.kl, "ratio_clip_min": 0.2, "ratio_clip_max": 0.2},
        "policy": pcfg,
    }
    torch.manual_seed(0)
    worker = PolicyWorker(pcfg, model_cfg=mcfg, pstate=ps, seed=1234)
    n_prompts = prompts_global * (args.warmup + args.steps + 1)
    ds = SyntheticPromptDataset(n_prompts, args.min_prompt, args.max_prompt, mcfg.vocab_size, seed=7)
    dl = StatefulDataLoader(ds, prompts_global, shuffle=False, shard_rank=ps.dp_rank, num_shards=ps.dp_size)
    env = {"synthetic": HashRewardEnvironment({"seed": 0})}

    step_log: list[dict] = []

    def cb(step, m):
        step_log.append({k: v for k, v in m.items() if isinstance(v, (int, float))})

    state = GRPOSaveState.default()
    # ---------------- warm-up (untimed) ----------------
    state = grpo_train(worker, iter_epochs(dl), env, cfg, save_state=state, max_steps=args.warmup, step_callback=cb)
    # ---------------- timed region ----------------
    clocks = ClockSampler([int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
                          or list(range(args.gpus))) if ps.rank == 0 else None
    if clocks:
        clocks.start()
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = _ext.launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record()
    n_before = len(step_log)
    state = grpo_train(worker, iter_epochs(dl), env, cfg, save_state=state, max_steps=args.warmup + args.steps,
                       step_callback=cb)
    ev1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if dist.is_initialized():
        dist.barrier()
    launches = _ext.launch_count() - launches0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    dev_s = max_over_ranks(dev_s)
    wall = max_over_ranks(wall)
    clk = clocks.stop() if clocks else None
    timed = step_log[n_before:]
    tokens = sum(s["total_tokens"] for s in timed)
    gen_tokens = sum(s["generated_tokens"] for s in timed)
    prompt_bytes = (tokens - gen_tokens) / max(1, ps.dp_size) * 8 / max(1, len(timed))  # int64 prompt ids per rank
    if ps.rank == 0:
        value = tokens / dev_s
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_s / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": f"synthetic prompts (uniform token ids, lengths U[{args.min_prompt},{args.max_prompt}]), "
                    "random-init weights, "
                    "seeded-hash reward",
            "config": {"model": pre["model_label"] + ("" if not args.layers else f" ({args.layers} layers: INVALID)"),
                       "global_batch": prompts_global * G, "seq_len": max_len,
                       "parallelism": f"tp{tp}dp{ps.dp_size}" + (f"ep{ep}" if ep > 1 else ""),
                       "rollout_tp": args.gen_tp or tp, "preset": args.preset,
                       "activation_checkpointing": pcfg["megatron_cfg"]["activation_checkpointing"], "prompts_per_step": prompts_global,
                       "generations_per_prompt": G, "max_new_tokens": args.max_new, "kl_penalty": args.kl,
                       "l2": "working set (16 GB bf16 weights + KV cache) far above the 126 MB L2; no flush needed",
                       "mean_gen_tokens": gen_tokens / max(1, len(timed)) / (prompts_global * G),
                       # one optimizer step per rollout batch: the "previous policy" logprobs equal the
                       # training forward's own, so that separate pass is folded into training
                       "prev_logprobs_from_train_forward": bool(cfg["grpo"].get("reuse_train_logprobs_as_prev", True)),
                       "reference_logprobs_pass": args.kl > 0,
                       "refit_kind": ("in-place: rollout reads the trained bf16 weights (same TP layout)"
                                      if (args.gen_tp or tp) == tp else
                                      f"reshard TP{tp}->TP{args.gen_tp} over NVLink peer loads"),
                       "eos_ignored": True},
            "e2e": {"value": round(tokens / wall, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(prompt_bytes), "d2h_bytes_per_step": 4 * len(timed) // max(1, len(timed))},
            "gpu_launches": int(launches),
            "clocks": clk,
            "step_breakdown_s": {k: round(sum(s.get(k, 0.0) for s in timed) / max(1, len(timed)), 3)
                                 for k in ("timing/generation", "timing/policy_and_reference_logprobs",
                                           "timing/policy_training", "timing/weight_sync", "timing/data_processing")},
            "gen_kl_error": timed[-1].get("gen_kl_error") if timed else None,
        }
        print(json.dumps(line), flush=True)
    shutdown(worker)


def shutdown(worker) -> None:
    """Tear down in an order that cannot hang, then return so the interpreter exits
    normally (its exit handlers run).  CUDA graphs that captured NCCL collectives are
    released before the process group.  A daemon watchdog ends the process only if
    teardown itself stalls; the result line is printed before this runs."""
    import gc

    import torch
    import torch.distributed as dist

    watchdog = threading.Timer(120.0, lambda: os._exit(3))
    watchdog.daemon = True
    watchdog.start()
    worker.shutdown()
    gc.collect()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    watchdog.cancel()


def iter_epochs(dl):
    """Endless iterator over a StatefulDataLoader (keeps its position)."""

    class _It:
        def __iter__(self):
            while True:
                yielded = False
                for b in dl:
                    yielded = True
                    yield b
                if not yielded:
                    return

    return _It()


if __name__ == "__main__":
    main()
