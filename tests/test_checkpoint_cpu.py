"""Checkpoint manager with asynchronous torch_dist weight writes: the step
directory is published only after the background write finishes, and the run
resumes from it (CPU)."""

from __future__ import annotations

import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_grpo_async_torch_dist_checkpoint_resumes(tmp_path):
    from examples.run_grpo import main
    from rl_b200.models.megatron_ckpt import is_torch_dist_checkpoint

    ck = str(tmp_path / "ckpt")
    args = ["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
            "logger.log_dir=" + str(tmp_path / "logs"), "logger.stdout=false", "checkpointing.enabled=true",
            f"++checkpointing.checkpoint_dir={ck}", "++checkpointing.save_period=2",
            "++checkpointing.model_save_format=torch_dist", "++checkpointing.save_optimizer=true",
            "++policy.megatron_cfg.checkpoint.async_save=true"]
    state = main(args + ["grpo.max_num_steps=2"])
    assert state["current_step"] == 2
    weights = os.path.join(ck, "step_2", "policy", "weights")
    assert is_torch_dist_checkpoint(weights)
    assert not os.path.exists(os.path.join(ck, "tmp_step_2"))
    state = main(args + ["grpo.max_num_steps=3"])
    assert state["current_step"] == 3
