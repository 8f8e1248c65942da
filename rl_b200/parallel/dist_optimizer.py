"""Distributed AdamW over the model's flat parameter buffer.

Equivalent of MCore's DistributedOptimizer with ``use_distributed_optimizer: true``
and ``data_parallel_sharding_strategy: optim_grads_params``
(``examples/configs/grpo_math_1B.yaml:225,244``; native component N13):

* gradients accumulate (fp32) in one flat ``main_grad`` buffer whose views are
  attached to the parameters (``rl_b200.ops.linear`` adds into them);
* ``step()``: reduce-scatter the flat gradient over the DP(xCP) group so every
  rank owns ``1/dp`` of it, compute the global grad norm (squares summed over
  the shard, then over DP and TP groups), run ONE fused AdamW launch over the
  shard (which also writes the bf16 parameters), and all-gather the bf16
  parameter shards back into the flat buffer;
* master weights / Adam moments exist only for the local shard
  (``12 bytes x params / dp`` per rank).

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
        # pad so the flat buffer splits evenly over DP ranks in 128-element units
        unit = 128 * self.dp
        self.padded = (n + unit - 1) // unit * unit
        if self.padded != n:
            pad = torch.zeros(self.padded - n, dtype=flat.dtype, device=flat.device)
            # re-home the flat buffer into a padded allocation (parameters keep their views)
            big = torch.cat([flat.detach(), pad])
            self._rehome(big)
        self.shard = self.padded // self.dp
        lo = self.dp_rank * self.shard
        self.lo, self.hi = lo, lo + self.shard
        dev = flat.device
        self.main_grad = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        self.master = model.flat_param[lo:lo + self.shard].float().clone()
        self.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.grad_shard = self.main_grad[lo:lo + self.shard] if self.dp == 1 else \
            torch.zeros(self.shard, dtype=torch.float32, device=dev)
        # weight-decay mask over the shard (norm weights / biases are excluded)
        self.wd_mask = torch.ones(self.shard, dtype=torch.float32, device=dev)
        self.replicated_mask = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        for sp, p in model.named_flat_params():
            a, b = max(sp.offset, lo), min(sp.offset + sp.numel, lo + self.shard)
            if a < b:
                if sp.no_weight_decay:
                    self.wd_mask[a - lo:b - lo] = 0.0
                if sp.tp_dim is None and sp.ep_dim is None:
                    self.replicated_mask[a - lo:b - lo] = 1.0
        self._attach_grads()
        self.step_count = 0
        self.last_grad_norm = 0.0

    def _rehome(self, big: torch.Tensor) -> None:
        m = self.model
        m.flat_param = big
        for sp, p in m.named_flat_params():
            p.data = big[sp.offset: sp.offset + sp.numel].view(sp.shape)

    def _attach_grads(self) -> None:
        for sp, p in self.model.named_flat_params():
            p.main_grad = self.main_grad[sp.offset: sp.offset + sp.numel].view(sp.shape)

    def zero_grad(self) -> None:
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

    @torch.no_grad()
    def step(self) -> dict:
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
        sq_rep = sum_of_squares(g * self.replicated_mask) if self.tp > 1 else None
        sq_all = sum_of_squares(g)
        if self.tp > 1:
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
        wd = self.weight_decay
        out = m.flat_param[self.lo:self.hi]
        if wd > 0 and float(self.wd_mask.min()) < 1.0:
            # decoupled decay only on masked-in params: apply decay separately
            self.master.mul_(1 - lr * wd * self.wd_mask)
            wd_eff = 0.0
        else:
            wd_eff = wd
        adamw_step(self.master, g, self.exp_avg, self.exp_avg_sq, lr, self.beta1, self.beta2, self.eps, wd_eff,
                   self.step_count, grad_scale=scale, param_out=out)
        if self.dp > 1:
            dist.all_gather_into_tensor(m.flat_param, out.clone(), group=self.dp_group)
        self.zero_grad()
        return {"grad_norm": norm, "lr": lr}

    def current_lr(self) -> float:
        return self.scheduler.lr_at(max(0, self.step_count - 1))

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
        with torch.no_grad():
            self.model.flat_param[self.lo:self.hi].copy_(self.master.to(self.model.flat_param.dtype))
            if self.dp > 1:
                dist.all_gather_into_tensor(self.model.flat_param, self.model.flat_param[self.lo:self.hi].clone(),
                                            group=self.dp_group)

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
