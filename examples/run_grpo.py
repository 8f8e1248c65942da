#!/usr/bin/env python
"""GRPO entry point (reference: ``examples/run_grpo.py:66``).

    python examples/run_grpo.py --config examples/configs/grpo_tiny_cpu.yaml [key=value ...]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/run_grpo.py --config ...

Loads the YAML (``defaults`` inheritance, ``${...}`` interpolation, Hydra-style
overrides), initialises the process groups from the torchrun environment
(TP / CP / EP sizes from ``policy.megatron_cfg``), builds the policy worker,
the sharded prompt loader and the environments, and runs ``grpo_train`` with
checkpointing and logging.  Resumes from the latest checkpoint when present.

Data: a ``data.train`` block (the reference's schema: dataset names or local
files, processors, prompt files, ``env_name`` per dataset) is tokenised with
``policy.tokenizer`` (a local tokenizer directory, or ``name: byte``) and
served with its environments through ``setup_response_data``; without one, the
prompts are synthetic token ids (``num_prompts``, ``min/max_prompt_len``) and
the environments come from the ``env:`` block.
"""

from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def build_envs(env_cfg: dict) -> dict:
    from rl_b200.environments.math_environment import MathEnvironment
    from rl_b200.environments.synthetic import EvenTokenEnvironment, HashRewardEnvironment

    envs = {}
    for task, c in (env_cfg or {}).items():
        kind = (c or {}).get("kind", task)
        if kind in ("hash", "synthetic"):
            envs[task] = HashRewardEnvironment(c)
        elif kind == "even":
            envs[task] = EvenTokenEnvironment(c)
        elif kind == "math":
            envs[task] = MathEnvironment(c)
        else:
            from rl_b200.environments.registry import make_environment

            envs[task] = make_environment(kind, c)
    return envs


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default=os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"))
    ap.add_argument("--role", default="trainer", choices=["trainer", "generator"],
                    help="with policy.generation.colocated.enabled=false: this process trains (and hosts the "
                         "data plane) or serves generation")
    args, overrides = ap.parse_known_args(argv)
    from rl_b200.algorithms.grpo import GRPOSaveState, grpo_train
    from rl_b200.data.datasets import StatefulDataLoader, SyntheticPromptDataset
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
    mcfg = get_model_config(cfg["policy"]["model_name"])
    d = cfg.get("data", {}) or {}
    seed = int(cfg["grpo"].get("seed", 0))
    tokenizer, val_dl, val_envs = None, None, None
    if d.get("train"):
        from rl_b200.data.tokenizer import get_tokenizer
        from rl_b200.data.utils import setup_response_data

        tokenizer = get_tokenizer(cfg["policy"].get("tokenizer") or {"name": cfg["policy"]["model_name"]})
        gen = cfg["policy"].setdefault("generation", {})
        gen.setdefault("pad_token_id", tokenizer.pad_token_id)
        if gen.get("stop_token_ids") is None:
            gen["stop_token_ids"] = [tokenizer.eos_token_id]
        ds, val_ds, envs, val_envs = setup_response_data(tokenizer, d, cfg.get("env", {}))
        if val_ds is not None:
            val_bs = int(cfg["grpo"].get("val_batch_size", cfg["grpo"]["num_prompts_per_step"]))
            val_bs = max(ps.dp_size, val_bs - val_bs % ps.dp_size)
            val_dl = StatefulDataLoader(val_ds, val_bs, shuffle=False, drop_last=False, shard_rank=ps.dp_rank,
                                        num_shards=ps.dp_size)
    else:
        task = next(iter(cfg.get("env", {"synthetic": {}})))
        ds = SyntheticPromptDataset(int(d.get("num_prompts", 1024)), int(d.get("min_prompt_len", 16)),
                                    int(d.get("max_prompt_len", 64)), mcfg.vocab_size, seed=seed, task_name=task)
        envs = build_envs(cfg.get("env", {}))
    dl = StatefulDataLoader(ds, int(cfg["grpo"]["num_prompts_per_step"]), shuffle=bool(d.get("shuffle", True)),
                            seed=seed, shard_rank=ps.dp_rank, num_shards=ps.dp_size)
    policy = PolicyWorker(cfg["policy"], model_cfg=mcfg, pstate=ps, seed=seed)
    ck = CheckpointManager(cfg.get("checkpointing", {})) if cfg.get("checkpointing", {}).get("enabled") else None
    state = GRPOSaveState.default()
    if ck is not None and ck.get_latest_checkpoint_path():
        paths = ck.get_resume_paths()
        info = ck.load_training_info(paths["root"])
        policy.load_checkpoint(paths["policy_weights"], paths["policy_optimizer"])
        if os.path.exists(paths["dataloader"]):
            import torch

            dl.load_state_dict(torch.load(paths["dataloader"]))
        state.update({k: info[k] for k in state if k in info})
    logger = Logger(cfg.get("logger", {}))
    logger.log_hyperparams(cfg)
    colo = (cfg["policy"].get("generation") or {}).get("colocated") or {}
    if not colo.get("enabled", True):
        state = _run_noncolocated(args.role, cfg, policy, dl, envs, logger, tokenizer)
    elif (cfg["grpo"].get("single_controller") or {}).get("enabled", False):
        from rl_b200.algorithms.single_controller import single_controller_train

        state = single_controller_train(policy, dl, envs, cfg, logger=logger, checkpointer=ck, save_state=state)
    elif (cfg["grpo"].get("async_grpo") or {}).get("enabled", False):
        from rl_b200.algorithms.async_grpo import async_grpo_train, restore_replay_buffer, restore_rollout_recovery

        buf, ledger = None, None
        if ck is not None and ck.get_latest_checkpoint_path():
            ledger = restore_rollout_recovery(ck.get_latest_checkpoint_path())
            acfg = cfg["grpo"].get("async_grpo") or {}
            n_groups = max(1, int(cfg["grpo"]["num_prompts_per_step"]) // max(1, ps.dp_size))
            age = int(acfg.get("max_trajectory_age_steps", 1))
            buf = restore_replay_buffer(ck.get_latest_checkpoint_path(), n_groups, n_groups * (age + 1) * 2,
                                        acfg.get("load_replay_buffer"))
        state = async_grpo_train(policy, dl, envs, cfg, logger=logger, checkpointer=ck, save_state=state,
                                 replay_buffer=buf, rollout_ledger=ledger)
    else:
        encode = (lambda text: tokenizer(text, add_special_tokens=False)["input_ids"]) if tokenizer else None
        state = grpo_train(policy, dl, envs, cfg, logger=logger, checkpointer=ck, save_state=state,
                           val_dataloader=val_dl, val_task_to_env=val_envs, tokenizer=encode)
    logger.close()
    policy.shutdown()  # waits for a background checkpoint write
    if ck is not None:
        ck.wait()  # and for the publication of its step directory
    return state


def _run_noncolocated(role: str, cfg: dict, policy, dl, envs, logger, tokenizer):
    """Trainer or generator of non-colocated GRPO: both processes run this entry
    point with the same config (``policy.generation.colocated``: ``host``,
    ``data_plane_port``, ``refit_port``, ``lead``), the trainer with ``--role trainer``."""
    from rl_b200.algorithms.grpo import GRPOSaveState
    from rl_b200.algorithms.noncolocated import noncolocated_grpo_train, serve_generation
    from rl_b200.data_plane.planes import StoreDataPlane
    from rl_b200.distributed.stateless_group import StatelessProcessGroup
    from rl_b200.weight_sync.broadcast import PackedBroadcastSynchronizer

    colo = cfg["policy"]["generation"]["colocated"]
    host = str(colo.get("host", "127.0.0.1"))
    trainer = role == "trainer"
    plane = StoreDataPlane(host=host, port=int(colo.get("data_plane_port", 29650)), is_master=trainer)
    group = StatelessProcessGroup(host, int(colo.get("refit_port", 29651)), 0 if trainer else 1, 2,
                                  timeout_s=float(colo.get("timeout_s", 600)))
    sync = PackedBroadcastSynchronizer(policy.model.flat_param if trainer else policy.gen_model.flat_param, group,
                                       src=0)
    state = GRPOSaveState.default()
    if trainer:
        hist = noncolocated_grpo_train(policy, dl, cfg, plane, sync, logger=logger)
        state["current_step"] = len(hist)
    else:
        state["current_step"] = serve_generation(policy, cfg, plane, sync, envs, tokenizer=tokenizer)
    group.barrier()
    return state


if __name__ == "__main__":
    main()
