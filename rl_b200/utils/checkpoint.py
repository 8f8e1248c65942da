"""Checkpoint directory management (reference: ``CheckpointManager``,
``nemo_rl/utils/checkpoint.py:259``; ``get_resume_paths`` ``:320``,
``init_tmp_checkpoint`` ``:379``, ``begin_finalization`` ``:436``,
``get_best_checkpoint_path`` ``:635``).

Layout::

    checkpoint_dir/
        step_N/
            training_info.json    loop state (step, epoch, consumed samples, metrics)
            config.yaml           the resolved run config
            policy/weights/       model weights (HF safetensors or sharded dist format)
            policy/optimizer/     optimizer shards
            train_dataloader.pt   dataloader position

A checkpoint is written into ``tmp_step_N`` and published by an atomic rename,
so a crash never leaves a half-written ``step_N``.  After publishing, only the
``keep_top_k`` best checkpoints by ``metric_name`` (``"train:loss"`` /
``"val:accuracy"``; ``higher_is_better``) plus the latest one are kept.
Finalisation (rename + pruning) can run on a background thread.
"""

from __future__ import annotations

import glob
import contextlib
import json
import os
import re
import shutil
import threading
from typing import Any, Optional

import yaml

__all__ = ["CheckpointManager", "DEFAULT_CHECKPOINT_CONFIG"]

DEFAULT_CHECKPOINT_CONFIG = {
    "enabled": True,
    "checkpoint_dir": "results/grpo",
    "metric_name": None,
    "higher_is_better": True,
    "keep_top_k": None,
    "save_period": 10,
    "checkpoint_must_save_by": None,
    "save_optimizer": True,
    "async_finalize": False,
    "model_save_format": "safetensors",   # "safetensors" (HF) or "torch_dist" (sharded)
}

_STEP_RE = re.compile(r"^step_(\d+)$")


class CheckpointManager:
    def __init__(self, config: Optional[dict] = None):
        c = dict(DEFAULT_CHECKPOINT_CONFIG)
        c.update(config or {})
        self.cfg = c
        self.checkpoint_dir = c["checkpoint_dir"]
        self.metric_name = c.get("metric_name")
        self.higher_is_better = bool(c.get("higher_is_better", True))
        self.keep_top_k = c.get("keep_top_k")
        self.save_period = int(c.get("save_period") or 0)
        self._thread: Optional[threading.Thread] = None

    # --------------------------------------------------------------- paths
    def step_dir(self, step: int) -> str:
        return os.path.join(self.checkpoint_dir, f"step_{step}")

    def tmp_dir(self, step: int) -> str:
        return os.path.join(self.checkpoint_dir, f"tmp_step_{step}")

    def list_steps(self) -> list[int]:
        if not os.path.isdir(self.checkpoint_dir):
            return []
        out = []
        for name in os.listdir(self.checkpoint_dir):
            m = _STEP_RE.match(name)
            if m and os.path.isfile(os.path.join(self.checkpoint_dir, name, "training_info.json")):
                out.append(int(m.group(1)))
        return sorted(out)

    def get_latest_checkpoint_path(self) -> Optional[str]:
        steps = self.list_steps()
        return self.step_dir(steps[-1]) if steps else None

    def get_resume_paths(self) -> dict:
        latest = self.get_latest_checkpoint_path()
        if latest is None:
            return {}
        return {"root": latest, "policy_weights": os.path.join(latest, "policy", "weights"),
                "policy_optimizer": os.path.join(latest, "policy", "optimizer"),
                "dataloader": os.path.join(latest, "train_dataloader.pt")}

    @staticmethod
    def load_training_info(path: Optional[str]) -> Optional[dict]:
        if path is None:
            return None
        with open(os.path.join(path, "training_info.json")) as f:
            return json.load(f)

    def deadline_reached(self) -> bool:
        """Mark a finished iteration; True when the next one would run past
        ``checkpoint_must_save_by`` (agreed over all ranks), so the loop saves
        and stops.  Reference: ``TimeoutChecker`` use in the training loops."""
        if not self.cfg.get("checkpoint_must_save_by"):
            return False
        if getattr(self, "_timeout", None) is None:
            from rl_b200.utils.timer import TimeoutChecker

            self._timeout = TimeoutChecker(self.cfg["checkpoint_must_save_by"])
            self._timeout.start_iterations()
            return False
        self._timeout.mark_iteration()
        hit = self._timeout.check_save()
        import torch
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_world_size() > 1:
            dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" \
                else torch.device("cpu")
            t = torch.tensor([1.0 if hit else 0.0], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            hit = bool(t.item() > 0)
        return hit

    def should_save(self, step: int) -> bool:
        return bool(self.cfg.get("enabled", True)) and self.save_period > 0 and step % self.save_period == 0

    # --------------------------------------------------------------- write
    def init_tmp_checkpoint(self, step: int, training_info: dict, run_config: Optional[dict] = None) -> str:
        self.wait()
        tmp = self.tmp_dir(step)
        if os.path.exists(tmp):
            shutil.rmtree(tmp)
        os.makedirs(os.path.join(tmp, "policy"), exist_ok=True)
        with open(os.path.join(tmp, "training_info.json"), "w") as f:
            json.dump(_jsonable(training_info), f, indent=2)
        if run_config is not None:
            with open(os.path.join(tmp, "config.yaml"), "w") as f:
                yaml.safe_dump(_jsonable(run_config), f, sort_keys=False)
        return tmp

    def finalize_checkpoint(self, tmp_path: str, wait_fn=None) -> str:
        """Publish ``tmp_step_N`` as ``step_N`` (atomic rename) and prune.  With
        ``wait_fn`` (the policy's ``finalize_async_save``: background weight writes
        still running) the rename happens on a background thread after it returns.
        With ``self.telemetry`` set (the loop's recorder) the publication is a
        ``checkpoint_finalize`` span in the caller's trace."""
        from rl_b200.utils.telemetry import current_trace_carrier, remote_trace_context

        carrier = current_trace_carrier()  # the finalize thread's spans stay in the caller's trace
        tele = getattr(self, "telemetry", None)

        def work():
            with remote_trace_context(carrier), (tele.span("checkpoint_finalize") if tele is not None
                                                 else contextlib.nullcontext()):
                _publish()

        def _publish():
            if wait_fn is not None:
                wait_fn()
            step = int(os.path.basename(tmp_path).split("_")[-1])
            final = self.step_dir(step)
            if os.path.exists(final):
                shutil.rmtree(final)
            os.replace(tmp_path, final)
            self.remove_old_checkpoints()

        if self.cfg.get("async_finalize") or wait_fn is not None:
            self._thread = threading.Thread(target=work, daemon=True)
            self._thread.start()
        else:
            work()
        return self.step_dir(int(os.path.basename(tmp_path).split("_")[-1]))

    begin_finalization = finalize_checkpoint

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None

    def _metric(self, step: int) -> Optional[float]:
        if not self.metric_name:
            return None
        info = self.load_training_info(self.step_dir(step)) or {}
        key = self.metric_name
        if key in info:
            return info[key]
        prefix, _, name = key.partition(":")
        return (info.get(prefix) or {}).get(name) if isinstance(info.get(prefix), dict) else info.get(name)

    def remove_old_checkpoints(self) -> None:
        if not self.keep_top_k:
            return
        steps = self.list_steps()
        if len(steps) <= int(self.keep_top_k):
            return
        latest = steps[-1]
        scored = [(self._metric(s), s) for s in steps]
        if all(v is None for v, _ in scored):
            keep = set(steps[-int(self.keep_top_k):])
        else:
            ranked = sorted((x for x in scored if x[0] is not None), key=lambda x: x[0],
                            reverse=self.higher_is_better)
            keep = {s for _, s in ranked[: int(self.keep_top_k)]}
        keep.add(latest)
        for s in steps:
            if s not in keep:
                shutil.rmtree(self.step_dir(s), ignore_errors=True)

    def get_best_checkpoint_path(self) -> Optional[str]:
        steps = self.list_steps()
        scored = [(self._metric(s), s) for s in steps if self._metric(s) is not None]
        if not scored:
            return self.get_latest_checkpoint_path()
        best = sorted(scored, key=lambda x: x[0], reverse=self.higher_is_better)[0][1]
        return self.step_dir(best)

    # ------------------------------------------------------ loop integration
    def save(self, policy, state: dict, dataloader=None, metrics: Optional[dict] = None, step: Optional[int] = None,
             run_config: Optional[dict] = None, rank_files: Optional[dict] = None) -> str:
        """Full checkpoint of a training loop (weights, optimizer, loop state).
        ``rank_files``: ``{file name: object}`` this rank writes with ``torch.save``
        into the checkpoint directory (per-rank state such as an async replay buffer)."""
        import torch
        import torch.distributed as dist

        step = int(step if step is not None else state.get("current_step", 0))
        rank0 = (not dist.is_initialized()) or dist.get_rank() == 0
        info = dict(state)
        if metrics:
            info["train"] = {k: v for k, v in metrics.items() if isinstance(v, (int, float))}
        tmp = self.init_tmp_checkpoint(step, info, run_config) if rank0 else self.tmp_dir(step)
        if dist.is_initialized():
            dist.barrier()
        policy.save_checkpoint(os.path.join(tmp, "policy", "weights"),
                               os.path.join(tmp, "policy", "optimizer") if self.cfg.get("save_optimizer") else None,
                               fmt=self.cfg.get("model_save_format", "safetensors"))
        if dataloader is not None and rank0 and hasattr(dataloader, "state_dict"):
            torch.save(dataloader.state_dict(), os.path.join(tmp, "train_dataloader.pt"))
        for name, obj in (rank_files or {}).items():
            torch.save(obj, os.path.join(tmp, name))
        if dist.is_initialized():
            dist.barrier()
        pending = getattr(policy, "poll_async_save", None)
        wait_fn = policy.finalize_async_save if pending is not None and not pending() else None
        if rank0:
            return self.finalize_checkpoint(tmp, wait_fn=wait_fn)
        return self.step_dir(step)


def _jsonable(x: Any) -> Any:
    if isinstance(x, dict):
        return {str(k): _jsonable(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_jsonable(v) for v in x]
    if isinstance(x, (int, float, str, bool)) or x is None:
        return x
    try:
        return float(x)
    except (TypeError, ValueError):
        return str(x)
