"""Distributed AdamW over the model's flat parameter buffer.

Equivalent of MCore's DistributedOptimizer with ``use_distributed_optimizer: true``
and ``data_parallel_sharding_strategy: optim_grads_params``
(``examples/configs/grpo_math_1B.yaml:225,244``; native component N13):

* gradients accumulate (fp32) in one flat ``main_grad`` buffer whose views are
  attached to the parameters (``rl_b200.ops.linear`` adds into them);
* ``step()``: reduce-scatter the flat gradient over the DP(xCP) group so every
  rank owns ``1/dp`` of it, compute the global grad norm (squares summed over
  the shard, then over DP and TP groups), run the fused AdamW kernel over the
  shard (which also writes the bf16 parameters) and all-gather the bf16
  parameter shards back into the flat buffer;
* master weights / Adam moments exist only for the local shard
  (``12 bytes x params / dp`` per rank); no other shard-sized state is kept
  (weight-decay and TP-replication classes are contiguous ranges).
* ``release_grad_buffer()`` frees the fp32 gradient buffer between training
  phases (the colocated rollout needs that HBM for its KV cache).

The reduce-scatter / all-gather here use NCCL; ``rl_b200.parallel.fused``
provides the peer-memory kernels that fuse them with the cast/scale/Adam work.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from rl_b200.ops.optim import adamw_step, sum_of_squares

__all__ = ["FlatAdamW", "LRScheduler"]


class LRScheduler:
    """Warm-up + decay schedule.  Accepts either the reference's list of torch
    schedulers (LinearLR warm-up then ConstantLR, ``grpo_math_1B.yaml`` policy.scheduler)
    or the Megatron scheduler block (``lr_warmup_iters``, ``lr_decay_style``...)."""

    def __init__(self, base_lr: float, cfg=None, min_lr: float = 0.0):
        self.base_lr = base_lr
        self.min_lr = min_lr
        self.warmup_iters = 0
        self.start_factor = 1.0
        self.decay_style = "constant"
        self.decay_iters = 0
        self.warmup_init = None
        if isinstance(cfg, list):
            for item in cfg:
                if not isinstance(item, dict) or "name" not in item:
                    continue
                if item["name"].endswith("LinearLR"):
                    kw = item.get("kwargs", {})
                    self.start_factor = float(kw.get("start_factor", 1.0))
                    self.warmup_iters = int(kw.get("total_iters", 0))
                elif item["name"].endswith("CosineAnnealingLR"):
                    self.decay_style = "cosine"
                    self.decay_iters = int(item.get("kwargs", {}).get("T_max", 0))
        elif isinstance(cfg, dict):
            self.warmup_iters = int(cfg.get("lr_warmup_iters", 0))
            self.warmup_init = cfg.get("lr_warmup_init")
            self.decay_style = cfg.get("lr_decay_style", "constant")
            self.decay_iters = int(cfg.get("lr_decay_iters", 0) or 0)

    def lr_at(self, it: int) -> float:
        if self.warmup_iters > 0 and it < self.warmup_iters:
            if self.warmup_init is not None:
                w0 = float(self.warmup_init)
                return w0 + (self.base_lr - w0) * it / self.warmup_iters
            f = self.start_factor + (1.0 - self.start_factor) * it / self.warmup_iters
            return self.base_lr * f
        if self.decay_style == "cosine" and self.decay_iters > 0:
            t = min(1.0, (it - self.warmup_iters) / max(1, self.decay_iters - self.warmup_iters))
            return self.min_lr + 0.5 * (self.base_lr - self.min_lr) * (1 + math.cos(math.pi * t))
        if self.decay_style == "linear" and self.decay_iters > 0:
            t = min(1.0, (it - self.warmup_iters) / max(1, self.decay_iters - self.warmup_iters))
            return self.base_lr + (self.min_lr - self.base_lr) * t
        return self.base_lr


def _merge(ranges: list[tuple[int, int, bool]]) -> list[tuple[int, int, bool]]:
    out: list[tuple[int, int, bool]] = []
    for a, b, f in sorted(ranges):
        if out and out[-1][2] == f and out[-1][1] == a:
            out[-1] = (out[-1][0], b, f)
        else:
            out.append((a, b, f))
    return out


class FlatAdamW:
    def __init__(self, model, lr: float = 1e-5, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                 max_grad_norm: Optional[float] = 1.0, scheduler_cfg=None, min_lr: float = 0.0,
                 dp_group=None, tp_group=None, sequence_parallel: bool = False):
        self.model = model
        self.lr = lr
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.scheduler = LRScheduler(lr, scheduler_cfg, min_lr)
        self.dp_group = dp_group
        self.tp_group = tp_group
        self.sequence_parallel = sequence_parallel
        self.dp = dist.get_world_size(dp_group) if (dp_group is not None and dist.is_initialized()) else 1
        self.dp_rank = dist.get_rank(dp_group) if self.dp > 1 else 0
        self.tp = dist.get_world_size(tp_group) if (tp_group is not None and dist.is_initialized()) else 1
        flat = model.flat_param
        n = flat.numel()
        unit = 128 * self.dp  # shards are 128-element aligned
        self.padded = (n + unit - 1) // unit * unit
        if self.padded != n:
            big = torch.zeros(self.padded, dtype=flat.dtype, device=flat.device)
            big[:n].copy_(flat.detach())
            self._rehome(big)
            del flat
        self.shard = self.padded // self.dp
        lo = self.dp_rank * self.shard
        self.lo, self.hi = lo, lo + self.shard
        dev = model.flat_param.device
        self.device = dev
        self.master = torch.empty(self.shard, dtype=torch.float32, device=dev)
        self.master.copy_(model.flat_param[lo:lo + self.shard])
        self.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        # contiguous shard-local ranges: (start, end, weight-decayed) and (start, end, TP-replicated)
        wd_r, rep_r = [], []
        covered = 0
        for sp, p in model.named_flat_params():
            a, b = max(sp.offset, lo), min(sp.offset + sp.numel, lo + self.shard)
            if a < b:
                wd_r.append((a - lo, b - lo, not sp.no_weight_decay))
                rep_r.append((a - lo, b - lo, sp.tp_dim is None and sp.ep_dim is None))
        self.wd_ranges = _merge(wd_r)
        self.rep_ranges = [(a, b) for a, b, f in _merge(rep_r) if f]
        self.main_grad: Optional[torch.Tensor] = None
        self.grad_shard: Optional[torch.Tensor] = None
        self.ensure_grad_buffer()
        self.step_count = 0
        self.last_grad_norm = 0.0

    # -------------------------------------------------------------- buffers
    def _rehome(self, big: torch.Tensor) -> None:
        m = self.model
        m.flat_param = big
        for sp, p in m.named_flat_params():
            p.data = big[sp.offset: sp.offset + sp.numel].view(sp.shape)

    def ensure_grad_buffer(self) -> None:
        if self.main_grad is not None:
            return
        self.main_grad = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        if self.dp == 1:
            self.grad_shard = self.main_grad[self.lo:self.hi]
        else:
            self.grad_shard = torch.zeros(self.shard, dtype=torch.float32, device=self.device)
        for sp, p in self.model.named_flat_params():
            p.main_grad = self.main_grad[sp.offset: sp.offset + sp.numel].view(sp.shape)

    def release_grad_buffer(self) -> None:
        """Free the fp32 gradient buffers (re-created zeroed by ``ensure_grad_buffer``)."""
        for _, p in self.model.named_flat_params():
            p.main_grad = None
            p.grad = None
        self.main_grad = None
        self.grad_shard = None

    def zero_grad(self) -> None:
        if self.main_grad is not None:
            self.main_grad.zero_()
        for _, p in self.model.named_flat_params():
            p.grad = None

    def _fold_param_grads(self) -> None:
        """Parameters whose gradient autograd produced in ``.grad`` (embedding
        lookups, norms, routers) are folded into the flat fp32 buffer."""
        for _, p in self.model.named_flat_params():
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None

    # ----------------------------------------------------------------- step
    @torch.no_grad()
    def step(self) -> dict:
        self.ensure_grad_buffer()
        self._fold_param_grads()
        m = self.model
        if self.sequence_parallel and self.tp > 1:
            # replicated params saw different tokens on each TP rank under SP
            for sp, p in m.named_flat_params():
                if sp.tp_dim is None and sp.ep_dim is None:
                    dist.all_reduce(p.main_grad, group=self.tp_group)
        if self.dp > 1:
            # losses are normalised by GLOBAL token / sequence counts, so the
            # per-rank gradients are partial sums: reduce with SUM, not mean.
            dist.reduce_scatter_tensor(self.grad_shard, self.main_grad, group=self.dp_group)
        g = self.grad_shard
        # global grad norm: TP-sharded parts summed over TP; replicated parts counted once
        sq_all = sum_of_squares(g)
        if self.tp > 1:
            sq_rep = torch.zeros((), dtype=torch.float32, device=g.device)
            for a, b in self.rep_ranges:
                sq_rep = sq_rep + sum_of_squares(g[a:b])
            sq_shard = sq_all - sq_rep
            dist.all_reduce(sq_shard, group=self.tp_group)
            sq = sq_shard + sq_rep
        else:
            sq = sq_all
        if self.dp > 1:
            dist.all_reduce(sq, group=self.dp_group)
        norm = float(sq.sqrt())
        self.last_grad_norm = norm
        scale = 1.0
        if self.max_grad_norm and self.max_grad_norm > 0 and norm > self.max_grad_norm:
            scale = self.max_grad_norm / (norm + 1e-6)
        if not math.isfinite(norm):
            self.zero_grad()
            return {"grad_norm": norm, "lr": self.current_lr(), "skipped": 1.0}
        self.step_count += 1
        lr = self.scheduler.lr_at(self.step_count - 1)
        out = m.flat_param[self.lo:self.hi]
        for a, b, decayed in self.wd_ranges:
            adamw_step(self.master[a:b], g[a:b], self.exp_avg[a:b], self.exp_avg_sq[a:b], lr, self.beta1,
                       self.beta2, self.eps, self.weight_decay if decayed else 0.0, self.step_count,
                       grad_scale=scale, param_out=out[a:b])
        if self.dp > 1:
            dist.all_gather_into_tensor(m.flat_param, out.clone(), group=self.dp_group)
        self.zero_grad()
        return {"grad_norm": norm, "lr": lr}

    def current_lr(self) -> float:
        return self.scheduler.lr_at(max(0, self.step_count - 1))

    @torch.no_grad()
    def restore_params_from_master(self) -> None:
        """Rewrite the bf16 parameters from the fp32 master copy (after a weight swap)."""
        m = self.model
        m.flat_param[self.lo:self.hi].copy_(self.master)
        if self.dp > 1:
            dist.all_gather_into_tensor(m.flat_param, m.flat_param[self.lo:self.hi].clone(), group=self.dp_group)

    # ---------------------------------------------------------- state dict
    def state_dict(self) -> dict:
        return {"master": self.master.cpu(), "exp_avg": self.exp_avg.cpu(), "exp_avg_sq": self.exp_avg_sq.cpu(),
                "step": self.step_count, "lo": self.lo, "hi": self.hi, "padded": self.padded}

    def load_state_dict(self, sd: dict) -> None:
        if sd["lo"] != self.lo or sd["hi"] != self.hi:
            raise ValueError("optimizer shard layout mismatch (different DP size?)")
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.step_count = int(sd["step"])
        self.restore_params_from_master()

    def offload(self) -> None:
        for name in ("master", "exp_avg", "exp_avg_sq"):
            t = getattr(self, name)
            if t.is_cuda:
                setattr(self, name, t.cpu())

    def onload(self, device) -> None:
        for name in ("master", "exp_avg", "exp_avg_sq"):
            t = getattr(self, name)
            if not t.is_cuda:
                setattr(self, name, t.to(device))
