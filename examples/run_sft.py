#!/usr/bin/env python
"""SFT entry point (reference: ``examples/run_sft.py``).

    python examples/run_sft.py --config examples/configs/sft_tiny_cpu.yaml [key=value ...]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/run_sft.py --config ...

Loads the YAML like ``run_grpo.py``, builds the policy worker and the
``data.train`` / ``data.validation`` datasets (``processor: sft_processor`` for
chat rows; ``dataset_name: megatron_sft_packed`` for offline-packed Megatron SFT
files, which takes the policy's context-parallel size), and runs ``sft_train``
with checkpointing and logging.  Resumes from the latest checkpoint when present.
"""

from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=os.path.join(ROOT, "examples", "configs", "sft_tiny_cpu.yaml"))
    args, overrides = ap.parse_known_args(argv)
    import torch

    from rl_b200.algorithms.sft import sft_train
    from rl_b200.data.datasets import StatefulDataLoader
    from rl_b200.data.tokenizer import get_tokenizer
    from rl_b200.data.utils import setup_response_data
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed
    from rl_b200.utils.checkpoint import CheckpointManager
    from rl_b200.utils.config import load_config
    from rl_b200.utils.logger import Logger

    cfg = load_config(args.config, overrides)
    mc = cfg["policy"].get("megatron_cfg", {}) or {}
    cp = int(mc.get("context_parallel_size", 1))
    ps = init_distributed(tp=int(mc.get("tensor_model_parallel_size", 1)), cp=cp,
                          ep=int(mc.get("expert_model_parallel_size", 1)),
                          pp=int(mc.get("pipeline_model_parallel_size", 1)))
    scfg = cfg.setdefault("sft", {})
    seed = int(scfg.get("seed", 0))
    tokenizer = get_tokenizer(cfg["policy"].get("tokenizer") or {"name": cfg["policy"]["model_name"]})
    ds, val_ds = setup_response_data(tokenizer, cfg["data"], context_parallel_size=cp)
    gbs = int(cfg["policy"]["train_global_batch_size"])
    dl = StatefulDataLoader(ds, gbs, shuffle=bool(cfg["data"].get("shuffle", True)), seed=seed,
                            shard_rank=ps.dp_rank, num_shards=ps.dp_size)
    val_dl = None
    if val_ds is not None:
        vbs = int(scfg.get("val_global_batch_size", gbs))
        val_dl = StatefulDataLoader(val_ds, max(ps.dp_size, vbs - vbs % ps.dp_size), shuffle=False, drop_last=False,
                                    shard_rank=ps.dp_rank, num_shards=ps.dp_size)
    policy = PolicyWorker(cfg["policy"], model_cfg=get_model_config(cfg["policy"]["model_name"]), pstate=ps,
                          seed=seed)
    ck = CheckpointManager(cfg.get("checkpointing", {})) if cfg.get("checkpointing", {}).get("enabled") else None
    state = None
    if ck is not None and ck.get_latest_checkpoint_path():
        paths = ck.get_resume_paths()
        info = ck.load_training_info(paths["root"])
        policy.load_checkpoint(paths["policy_weights"], paths["policy_optimizer"])
        if os.path.exists(paths["dataloader"]):
            dl.load_state_dict(torch.load(paths["dataloader"]))
        state = {k: info[k] for k in ("current_step", "current_epoch", "total_steps") if k in info}
    logger = Logger(cfg.get("logger", {}))
    logger.log_hyperparams(cfg)
    state = sft_train(policy, dl, cfg, logger=logger, checkpointer=ck, save_state=state, val_dataloader=val_dl)
    logger.close()
    policy.shutdown()
    if ck is not None:
        ck.wait()
    return state


if __name__ == "__main__":
    main()
