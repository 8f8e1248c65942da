#!/usr/bin/env python
"""Evaluation entry point (reference: ``examples/run_eval.py``).

    python examples/run_eval.py --config examples/configs/eval_tiny_cpu.yaml [key=value ...]

Loads the YAML like ``run_grpo.py``, builds the policy worker (``policy.model_name``;
``checkpoint_path`` loads trained weights), the benchmark named by
``data.dataset_name`` (``setup_eval_data``: math / math500, gpqa / gpqa_diamond,
mmlu / mmlu_<LANG>, mmlu_pro, or a local CSV / JSON math set) and the ``env:``
block's environment, and reports ``eval.metric`` (``pass@k`` / ``cons@k``) with
``eval.num_tests_per_prompt`` samples per prompt.
"""

from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=os.path.join(ROOT, "examples", "configs", "eval_tiny_cpu.yaml"))
    args, overrides = ap.parse_known_args(argv)
    from examples.run_grpo import build_envs
    from rl_b200.data.datasets import StatefulDataLoader
    from rl_b200.data.eval_datasets import setup_eval_data
    from rl_b200.data.tokenizer import get_tokenizer
    from rl_b200.evals.eval import run_env_eval
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed
    from rl_b200.utils.config import load_config

    cfg = load_config(args.config, overrides)
    mc = cfg["policy"].get("megatron_cfg", {}) or {}
    ps = init_distributed(tp=int(mc.get("tensor_model_parallel_size", 1)))
    tokenizer = get_tokenizer(cfg["policy"].get("tokenizer") or {"name": cfg["policy"]["model_name"]})
    gen = cfg["policy"].setdefault("generation", {})
    gen.setdefault("pad_token_id", tokenizer.pad_token_id)
    if gen.get("stop_token_ids") is None:
        gen["stop_token_ids"] = [tokenizer.eos_token_id]
    ds, base = setup_eval_data(tokenizer, cfg["data"])
    ecfg = cfg.setdefault("eval", {})
    bs = int(ecfg.get("batch_size", 8))
    dl = StatefulDataLoader(ds, max(ps.dp_size, bs - bs % ps.dp_size), shuffle=False, drop_last=False,
                            shard_rank=ps.dp_rank, num_shards=ps.dp_size)
    policy = PolicyWorker(cfg["policy"], model_cfg=get_model_config(cfg["policy"]["model_name"]), pstate=ps,
                          seed=int(ecfg.get("seed", 0)))
    if cfg.get("checkpoint_path"):
        policy.load_checkpoint(cfg["checkpoint_path"], None)
    envs = build_envs(cfg.get("env", {}))
    env = envs.get(base.task_spec.task_name) or next(iter(envs.values()))
    encode = lambda text: tokenizer.encode(text, add_special_tokens=False)
    res = run_env_eval(policy, dl, {base.task_spec.task_name: env, "default": env}, cfg, tokenizer=encode)
    if ps.rank == 0:
        print({"dataset": cfg["data"]["dataset_name"], **res})
    policy.shutdown()
    return res


if __name__ == "__main__":
    main()
