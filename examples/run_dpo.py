#!/usr/bin/env python
"""DPO entry point (reference: ``examples/run_dpo.py``).

    python examples/run_dpo.py --config examples/configs/dpo_tiny_cpu.yaml [key=value ...]

Loads the YAML like ``run_grpo.py``, builds the policy worker and the
``data.train`` preference dataset (``load_preference_dataset``: HelpSteer3,
Tulu3Preference, BinaryPreferenceDataset, PreferenceDataset or a dotted class
path), tokenises its rows through ``preference_preprocessor`` and runs
``dpo_train`` (``dpo:`` block: ``reference_policy_kl_penalty``,
``preference_loss_weight``, ``sft_loss_weight``, ...) with logging.
"""

from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=os.path.join(ROOT, "examples", "configs", "dpo_tiny_cpu.yaml"))
    args, overrides = ap.parse_known_args(argv)
    from rl_b200.algorithms.dpo import dpo_train
    from rl_b200.data.datasets import StatefulDataLoader
    from rl_b200.data.preference_datasets import PreferenceSamples, load_preference_dataset
    from rl_b200.data.tokenizer import get_tokenizer
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed
    from rl_b200.utils.checkpoint import CheckpointManager
    from rl_b200.utils.config import load_config
    from rl_b200.utils.logger import Logger

    cfg = load_config(args.config, overrides)
    mc = cfg["policy"].get("megatron_cfg", {}) or {}
    ps = init_distributed(tp=int(mc.get("tensor_model_parallel_size", 1)), cp=int(mc.get("context_parallel_size", 1)),
                          ep=int(mc.get("expert_model_parallel_size", 1)),
                          pp=int(mc.get("pipeline_model_parallel_size", 1)))
    seed = int(cfg.setdefault("dpo", {}).get("seed", 0))
    tokenizer = get_tokenizer(cfg["policy"].get("tokenizer") or {"name": cfg["policy"]["model_name"]})
    data = cfg["data"]
    ds = load_preference_dataset(dict(data["train"]))
    samples = PreferenceSamples(ds, tokenizer, data.get("max_input_seq_length",
                                                        cfg["policy"]["max_total_sequence_length"]))
    # each sample is a chosen / rejected pair: a global batch of B rows holds B / 2 pairs
    pairs = max(1, int(cfg["policy"]["train_global_batch_size"]) // 2)
    dl = StatefulDataLoader(samples, pairs, shuffle=bool(data.get("shuffle", True)), seed=seed,
                            collate_fn=lambda b: b, shard_rank=ps.dp_rank, num_shards=ps.dp_size)
    policy = PolicyWorker(cfg["policy"], model_cfg=get_model_config(cfg["policy"]["model_name"]), pstate=ps,
                          seed=seed)
    ck = CheckpointManager(cfg.get("checkpointing", {})) if cfg.get("checkpointing", {}).get("enabled") else None
    logger = Logger(cfg.get("logger", {}))
    logger.log_hyperparams(cfg)
    state = dpo_train(policy, dl, cfg, logger=logger, checkpointer=ck)
    logger.close()
    policy.shutdown()
    if ck is not None:
        ck.wait()
    return state


if __name__ == "__main__":
    main()
