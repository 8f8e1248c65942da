"""Non-colocated GRPO (CPU): a trainer process and a generator process that
share only a TCPStore data plane and a two-member stateless group for the weight
broadcast; on-policy (lead 0) and one-step-ahead (lead 1) schedules end with the
generator holding exactly the trainer's weights."""

from __future__ import annotations

import multiprocessing as mp
import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(lead: int, steps: int = 3):
    from rl_b200.utils.config import load_config

    cfg = load_config(os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"), [])
    cfg["grpo"]["max_num_steps"] = steps
    cfg["policy"].setdefault("generation", {})["colocated"] = {"enabled": False, "lead": lead}
    return cfg


def _trainer(lead, plane_port, group_port, q):
    from rl_b200.algorithms.noncolocated import noncolocated_grpo_train
    from rl_b200.data.datasets import StatefulDataLoader, SyntheticPromptDataset
    from rl_b200.data_plane.planes import StoreDataPlane
    from rl_b200.distributed.stateless_group import StatelessProcessGroup
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.weight_sync.broadcast import PackedBroadcastSynchronizer

    cfg = _cfg(lead)
    plane = StoreDataPlane(host="127.0.0.1", port=plane_port, is_master=True)
    group = StatelessProcessGroup("127.0.0.1", group_port, 0, 2, backend="gloo", timeout_s=120)
    mcfg = get_model_config(cfg["policy"]["model_name"])
    w = PolicyWorker(cfg["policy"], model_cfg=mcfg, seed=0)
    ds = SyntheticPromptDataset(64, 16, 16, mcfg.vocab_size, seed=0, task_name="synthetic")
    dl = StatefulDataLoader(ds, int(cfg["grpo"]["num_prompts_per_step"]), shuffle=False)
    sync = PackedBroadcastSynchronizer(w.model.flat_param, group, src=0, bucket_bytes=1 << 16)
    hist = noncolocated_grpo_train(w, dl, cfg, plane, sync)
    q.put(("trainer", [h["loss"] for h in hist], w.model.flat_param.detach().clone()))
    group.barrier()


def _generator(lead, plane_port, group_port, q):
    from examples.run_grpo import build_envs
    from rl_b200.algorithms.noncolocated import serve_generation
    from rl_b200.data_plane.planes import StoreDataPlane
    from rl_b200.distributed.stateless_group import StatelessProcessGroup
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.weight_sync.broadcast import PackedBroadcastSynchronizer

    cfg = _cfg(lead)
    plane = StoreDataPlane(host="127.0.0.1", port=plane_port, is_master=False)
    group = StatelessProcessGroup("127.0.0.1", group_port, 1, 2, backend="gloo", timeout_s=120)
    w = PolicyWorker(cfg["policy"], model_cfg=get_model_config(cfg["policy"]["model_name"]), seed=123)
    sync = PackedBroadcastSynchronizer(w.model.flat_param, group, src=0, bucket_bytes=1 << 16)
    served = serve_generation(w, cfg, plane, sync, build_envs(cfg.get("env", {})))
    q.put(("generator", served, w.model.flat_param.detach().clone()))
    group.barrier()


@pytest.mark.parametrize("lead", [0, 1])
def test_noncolocated_trainer_and_generator(lead):
    from rl_b200.distributed.launch import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    pp, gp = free_port(), free_port()
    procs = [ctx.Process(target=_trainer, args=(lead, pp, gp, q)),
             ctx.Process(target=_generator, args=(lead, pp, gp, q))]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            role, a, flat = q.get(timeout=300)
            out[role] = (a, flat)
    finally:
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.terminate()
    losses, tflat = out["trainer"]
    served, gflat = out["generator"]
    assert len(losses) == 3 and served == 3
    assert all(torch.isfinite(torch.tensor(losses)))
    assert torch.equal(tflat, gflat)  # the generator holds the trained weights


def _role(role, pp, gp, q):
    from examples.run_grpo import main

    cfg = os.path.join(ROOT, "examples", "configs", "grpo_tiny_noncolocated_cpu.yaml")
    st = main(["--config", cfg, "--role", role, "logger.stdout=false",
               f"policy.generation.colocated.data_plane_port={pp}", f"policy.generation.colocated.refit_port={gp}",
               "grpo.max_num_steps=2", f"logger.log_dir=/tmp/rlb_noncolo_{role}_{pp}"])
    q.put((role, int(st["current_step"])))


def test_noncolocated_through_the_entry_point():
    from rl_b200.distributed.launch import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    pp, gp = free_port(), free_port()
    procs = [ctx.Process(target=_role, args=(r, pp, gp, q)) for r in ("trainer", "generator")]
    for p in procs:
        p.start()
    try:
        got = dict(q.get(timeout=300) for _ in range(2))
    finally:
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.terminate()
    assert got == {"trainer": 2, "generator": 2}
