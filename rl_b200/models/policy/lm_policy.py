"""``Policy``: the reference's policy facade over this rank's ``PolicyWorker``.

The reference drives one Ray actor per GPU from a single controller through a
``Policy`` object (``nemo_rl/models/policy/lm_policy.py``); here every rank runs
the same program (SPMD, one process per GPU), so the facade forwards each call
to the local worker, which performs the collectives with its peers.  Method
names and arguments follow the reference so algorithm code written against it
runs unchanged: ``train``, ``get_logprobs``, ``get_reference_policy_logprobs``,
``get_topk_logits``, ``generate``, ``score``, the generation / training /
refit lifecycle, ``calibrate_qkv_fp8_scales``, checkpoints and profiling.

Reference: ``nemo_rl/models/policy/lm_policy.py:539-1590`` (``Policy``) and
``nemo_rl/models/policy/interfaces.py:73-318`` (``PolicyInterface``).
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["Policy"]


class Policy:
    def __init__(self, worker=None, **worker_kwargs):
        """Wrap an existing ``PolicyWorker`` or build one from ``worker_kwargs``
        (``policy_cfg``, ``model_cfg``, ``pstate``, ``seed``, ...)."""
        if worker is None:
            from rl_b200.models.policy.worker import PolicyWorker

            worker = PolicyWorker(**worker_kwargs)
        self.worker = worker
        self.cfg = worker.cfg

    # ------------------------------------------------------------ topology
    @property
    def data_parallel_size(self) -> int:
        return self.worker.ps.dp_size

    def run_all_workers_single_data(self, method_name: str, *args, **kwargs) -> Any:
        """Call ``method_name`` on the worker (every rank does the same)."""
        return getattr(self.worker, method_name)(*args, **kwargs)

    def run_all_workers_multiple_data(self, method_name: str, *args, **kwargs) -> Any:
        return self.run_all_workers_single_data(method_name, *args, **kwargs)

    # ------------------------------------------------------------ compute
    def get_logprobs(self, data: BatchedDataDict, timer=None, **kw) -> BatchedDataDict:
        return self.worker.get_logprobs(data, **kw)

    def get_reference_policy_logprobs(self, data: BatchedDataDict, timer=None, **kw) -> BatchedDataDict:
        return self.worker.get_reference_policy_logprobs(data, **kw)

    @torch.no_grad()
    def get_topk_logits(self, data: BatchedDataDict, k: int, timer=None) -> BatchedDataDict:
        """Top-``k`` next-token logits per position (``topk_logits``,
        ``topk_indices`` ``[B, S, k]``; position i scores token i+1), as the
        reference's teacher for top-k distillation."""
        w = self.worker
        ids = data["input_ids"]
        B, S = ids.shape
        lengths = w._lengths(data)
        vals = torch.zeros(B, S, k, dtype=torch.float32)
        idx = torch.zeros(B, S, k, dtype=torch.int64)

        class _Logits:
            from rl_b200.algorithms.loss.interfaces import LossInputType as _LIT

            input_type = _LIT.LOGIT

        w.model.eval()
        try:
            for rows in w._plan(lengths, [r for r in range(B) if lengths[r] > 0], w.logprob_mb_tokens):
                if rows[0] < 0:
                    continue
                width = max(lengths[r] for r in rows)
                logits = w._loss_input(_Logits(), ids, lengths, rows, width, 1.0)  # [n, width-1, V]
                tv, ti = logits.float().topk(k, dim=-1)
                vals[torch.tensor(rows), : width - 1] = tv.cpu()
                idx[torch.tensor(rows), : width - 1] = ti.cpu()
        finally:
            w.model.train()
        return BatchedDataDict({"topk_logits": vals, "topk_indices": idx})

    def train(self, data: BatchedDataDict, loss_fn, eval_mode: bool = False, gbs: Optional[int] = None,
              mbs: Optional[int] = None, timer=None, **kw) -> dict:
        return self.worker.train(data, loss_fn, gbs=gbs, eval_mode=eval_mode, **kw)

    def generate(self, data: BatchedDataDict, greedy: bool = False, timer=None) -> BatchedDataDict:
        return self.worker.generate(data, greedy=greedy)

    def score(self, data: BatchedDataDict, timer=None) -> BatchedDataDict:
        """Reward-model scores: the value head at each sequence's last token."""
        vals = self.worker.get_values(data)["values"]
        lengths = torch.tensor(self.worker._lengths(data)).clamp_min(1)
        return BatchedDataDict({"scores": vals[torch.arange(vals.shape[0]), lengths - 1]})

    # ------------------------------------------------------------ lifecycle
    def prepare_for_generation(self, *args, **kwargs) -> bool:
        return self.worker.prepare_for_generation(*args, **kwargs)

    def finish_generation(self, *args, **kwargs) -> bool:
        return self.worker.finish_generation()

    def prepare_for_training(self, *args, **kwargs) -> None:
        self.worker.prepare_for_training()

    def prepare_for_lp_inference(self, keep_train_buffers: bool = False) -> None:
        self.worker.prepare_for_lp_inference()

    def finish_training(self, *args, **kwargs) -> None:
        """Training buffers stay resident between steps (colocated loop); nothing to release."""

    def finish_inference(self) -> None:
        """Log-prob passes hold no state to release."""

    def invalidate_kv_cache(self, *args, **kwargs) -> bool:
        return self.worker.engine.invalidate_kv_cache()

    # ---------------------------------------------------------------- refit
    def prepare_refit_info(self) -> Optional[dict[str, Any]]:
        """Name -> (shape, dtype) of the rollout parameters."""
        m = self.worker.gen_model
        return {sp.name: (tuple(sp.shape), m.dtype) for sp in m.specs}

    def refit(self) -> float:
        return self.worker.refit()

    def sync_params_before_refit(self) -> None:
        """The flat parameter buffer is already consistent after the optimizer step
        (the fused DP update all-gathers it), so there is nothing to synchronise."""

    def offload_before_refit(self) -> None:
        self.worker.offload_before_refit()

    def offload_after_refit(self) -> None:
        self.worker.offload_after_refit()

    @property
    def sharding_annotations(self):
        """``NamedSharding`` of the process grid (pipeline, data, context, tensor axes)."""
        from rl_b200.distributed.named_sharding import from_parallel_state

        return from_parallel_state(self.worker.ps)

    def recreate_worker(self, worker_idx: int = 0) -> None:
        """Rebuild this rank's rollout engine (the generation shard) in place and
        re-synchronise its weights; ``worker_idx`` is accepted for the reference's
        signature (one engine per rank here)."""
        self.worker.recreate_generation_engine()

    def offload_to_cpu(self) -> None:
        self.worker.offload_to_cpu()

    def onload(self) -> None:
        self.worker.onload()

    def calibrate_qkv_fp8_scales(self, data: BatchedDataDict, **kw) -> dict:
        return self.worker.calibrate_qkv_fp8_scales(data, **kw)

    def get_free_memory_bytes(self) -> int:
        if torch.cuda.is_available():
            return int(torch.cuda.mem_get_info()[0])
        return 0

    # ---------------------------------------------------------- checkpoints
    def save_checkpoint(self, weights_path: str, optimizer_path: Optional[str] = None, **kw) -> None:
        self.worker.save_checkpoint(weights_path, optimizer_path, **kw)

    def load_checkpoint(self, weights_path: str, optimizer_path: Optional[str] = None) -> None:
        self.worker.load_checkpoint(weights_path, optimizer_path)

    def finalize_async_save(self) -> None:
        self.worker.finalize_async_save()

    def poll_async_save(self) -> bool:
        return self.worker.poll_async_save()

    # ------------------------------------------------------------ profiling
    def start_gpu_profiling(self) -> None:
        if torch.cuda.is_available():
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStart()

    def stop_gpu_profiling(self) -> None:
        if torch.cuda.is_available():
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()

    def shutdown(self) -> bool:
        self.worker.shutdown()
        return True
