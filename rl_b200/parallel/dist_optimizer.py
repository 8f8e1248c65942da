"""Distributed AdamW over the model's flat parameter buffer.

Equivalent of MCore's DistributedOptimizer with ``use_distributed_optimizer: true``
and ``data_parallel_sharding_strategy: optim_grads_params``
(``examples/configs/grpo_math_1B.yaml:225,244``; native component N13):

* gradients accumulate (fp32) in one flat ``main_grad`` buffer whose views are
  attached to the parameters (``rl_b200.ops.linear`` adds into them);
* the flat buffer has up to two contiguous SEGMENTS - dense parameters, reduced
  over the data-parallel (x context-parallel) group, and MoE expert parameters,
  reduced over the expert-data-parallel group (ranks that hold the same experts);
* ``step()``: per segment, reduce-scatter the gradient so each rank owns
  ``1/group`` of it, compute the global grad norm (shard squares summed over the
  reduction group, TP-replicated parts counted once, expert parts summed over the
  EP group), run the fused AdamW kernel over the shard (which also writes the
  bf16 parameters) and all-gather the bf16 shards back into the flat buffer;
* master weights / Adam moments exist only for the local shards
  (``12 bytes x params / group`` per rank); no other shard-sized state is kept
  (weight-decay and TP-replication classes are contiguous ranges).

The reduce-scatter / all-gather here use NCCL; ``rl_b200.parallel.fused``
provides the peer-memory kernels that fuse them with the cast/scale/Adam work.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from rl_b200.ops._ext import ext

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


def _ws(group) -> int:
    return dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1


class _Segment:
    """A contiguous range of the flat buffer with one gradient-reduction group."""

    def __init__(self, lo: int, hi: int, group, norm_sum_group, expert: bool, replicated: bool = False):
        self.lo, self.hi = lo, hi            # global offsets in the flat buffer (padded)
        self.group = group
        self.n = _ws(group)
        self.rank = dist.get_rank(group) if self.n > 1 else 0
        self.norm_sum_group = norm_sum_group  # extra group the shard norm^2 is summed over
        self.expert = expert
        # replicated: gradients all-reduced and every rank steps the whole range
        # (Muon needs whole matrices); otherwise ZeRO-1 shards over the group
        self.sharded = self.n > 1 and not replicated
        size = hi - lo
        self.shard = size // self.n if self.sharded else size
        self.s_lo = lo + (self.rank * self.shard if self.sharded else 0)  # this rank's shard (global offsets)
        self.s_hi = self.s_lo + self.shard


class FlatAdamW:
    def __init__(self, model, lr: float = 1e-5, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                 max_grad_norm: Optional[float] = 1.0, scheduler_cfg=None, min_lr: float = 0.0,
                 dp_group=None, tp_group=None, sequence_parallel: bool = False, edp_group=None, ep_group=None,
                 symmetric=None, pp_group=None, muon=None):
        """``symmetric``: a ``rl_b200.parallel.symm.NodeSymmetric`` allocator.  When
        given (CUDA, every rank on one node) the fp32 gradient buffer and the bf16
        parameter buffer are symmetric memory and the dense data-parallel segment
        steps with the fused kernels of ``csrc/dp_optim.cu`` (reduce-scatter by
        peer loads + norm partials, then AdamW fused with the parameter all-gather
        by peer stores) instead of NCCL reduce-scatter / all-gather.
        ``pp_group``: under pipeline parallelism each stage steps its own layers;
        the gradient norm used for clipping is the whole model's (sum of squares
        over the stages).
        ``muon``: a ``rl_b200.parallel.muon.MuonConfig``; the linear layers'
        weights then step with Muon (momentum kept in ``exp_avg``) and the rest
        with AdamW, on replicated segments (gradients all-reduced over the
        data-parallel group, no optimizer-state sharding)."""
        self.model = model
        self.muon = muon
        self.symmetric = symmetric
        self.lr = lr
        self.beta1, self.beta2 = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self.max_grad_norm = max_grad_norm
        self.scheduler = LRScheduler(lr, scheduler_cfg, min_lr)
        self.dp_group = dp_group
        self.tp_group = tp_group
        self.pp_group = pp_group if _ws(pp_group) > 1 else None
        self.sequence_parallel = sequence_parallel
        self.tp = _ws(tp_group)
        self.dp = _ws(dp_group)
        dense_n = int(getattr(model, "expert_offset", model.flat_numel))
        expert_n = int(model.flat_numel) - dense_n
        u_d = 128 * max(1, _ws(dp_group))
        dense_pad = (dense_n + u_d - 1) // u_d * u_d
        rep = muon is not None
        segs = [_Segment(0, dense_pad, dp_group, None, False, replicated=rep)]
        total = dense_pad
        if expert_n > 0:
            g = edp_group if edp_group is not None else dp_group
            u_e = 128 * max(1, _ws(g))
            exp_pad = (expert_n + u_e - 1) // u_e * u_e
            segs.append(_Segment(dense_pad, dense_pad + exp_pad, g, ep_group, True, replicated=rep))
            total = dense_pad + exp_pad
        self.segments = segs
        self.padded = total
        self._relayout(dense_pad - dense_n)
        dev = model.flat_param.device
        self.device = dev
        for seg in self.segments:
            seg.master = torch.empty(seg.shard, dtype=torch.float32, device=dev)
            seg.master.copy_(model.flat_param[seg.s_lo:seg.s_hi])
            seg.exp_avg = torch.zeros(seg.shard, dtype=torch.float32, device=dev)
            seg.exp_avg_sq = torch.zeros(seg.shard, dtype=torch.float32, device=dev)
            wd_r, rep_r = [], []
            seg.muon_params = []
            from rl_b200.parallel.muon import is_muon_param

            for sp, p in model.named_flat_params():
                a, b = max(sp.offset, seg.s_lo), min(sp.offset + sp.numel, seg.s_hi)
                if a < b:
                    if muon is not None and is_muon_param(sp.name):
                        seg.muon_params.append((sp, a - seg.s_lo, b - seg.s_lo))
                    else:
                        wd_r.append((a - seg.s_lo, b - seg.s_lo, not sp.no_weight_decay))
                    # replicated over TP (every TP rank holds the same values): counted once
                    # in the norm; whole experts without an FFN split are replicated too
                    rep_r.append((a - seg.s_lo, b - seg.s_lo, sp.tp_dim is None))
            seg.wd_ranges = _merge(wd_r)
            seg.frozen_ranges = []
            seg.rep_ranges = [(a, b) for a, b, f in _merge(rep_r) if f]
            nd = [(a, b) for a, b, d in seg.wd_ranges if not d]
            seg.nodecay_dev = torch.tensor(nd if nd else [[seg.shard, seg.shard]], dtype=torch.int64,
                                           device=dev).view(-1, 2)
        self.main_grad: Optional[torch.Tensor] = None
        self.ensure_grad_buffer()
        self.step_count = 0
        self.last_grad_norm = 0.0
        self._ov = None            # reduction overlapped with the backward (setup_overlap)
        self._ov_active = False

    # ------------------------------------------------------- flat re-layout
    def _relayout(self, expert_shift: int) -> None:
        """Move the flat buffer into a ``self.padded`` allocation, shifting expert
        parameters behind the padded dense segment; parameters are rebound."""
        m = self.model
        old = m.flat_param
        if self.padded == old.numel() and expert_shift == 0:
            return
        alloc = getattr(m, "_flat_alloc", None)
        if alloc is not None:
            big = alloc(self.padded, old.dtype)
            big.zero_()
        else:
            big = torch.zeros(self.padded, dtype=old.dtype, device=old.device)
        for sp, p in m.named_flat_params():
            new_off = sp.offset + (expert_shift if sp.ep_dim is not None else 0)
            big[new_off:new_off + sp.numel].copy_(old[sp.offset:sp.offset + sp.numel])
            sp.offset = new_off
        m.flat_param = big
        for sp, p in m.named_flat_params():
            p.data = big[sp.offset: sp.offset + sp.numel].view(sp.shape)
        old_symm = getattr(old, "_symm", None)
        if old_symm is not None and self.symmetric is not None:
            self.symmetric.release(old_symm)
        if hasattr(m, "expert_offset"):
            m.expert_offset = self.segments[-1].lo if self.segments[-1].expert else self.padded
        del old

    # -------------------------------------------------------------- buffers
    def ensure_grad_buffer(self) -> None:
        if self.main_grad is not None:
            return
        if self.symmetric is not None:
            self._grad_symm = self.symmetric.alloc(self.padded * 4)
            self.main_grad = self._grad_symm.local_view(torch.float32, self.padded)
            self.main_grad.zero_()
        else:
            self.main_grad = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        for seg in self.segments:
            if not seg.sharded:
                seg.grad_shard = self.main_grad[seg.s_lo:seg.s_hi]
            else:
                seg.grad_shard = torch.zeros(seg.shard, dtype=torch.float32, device=self.device)
        for sp, p in self.model.named_flat_params():
            p.main_grad = self.main_grad[sp.offset: sp.offset + sp.numel].view(sp.shape)

    def release_grad_buffer(self) -> None:
        """Free the fp32 gradient buffers (re-created zeroed by ``ensure_grad_buffer``).
        A symmetric gradient buffer stays (its allocation is collective)."""
        if self.symmetric is not None:
            return
        for _, p in self.model.named_flat_params():
            p.main_grad = None
            p.grad = None
        self.main_grad = None
        for seg in self.segments:
            seg.grad_shard = None

    def zero_grad(self) -> None:
        if self.main_grad is not None:
            self.main_grad.zero_()
        for _, p in self.model.named_flat_params():
            p.grad = None

    def _fold_param_grads(self) -> None:
        """Parameters whose gradient autograd produced in ``.grad`` (routers,
        parameters outside the fused ops) are folded into the flat fp32 buffer."""
        for _, p in self.model.named_flat_params():
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None

    # ------------------------------------------------------------ freezing
    def freeze(self, pred) -> int:
        """Freeze the parameters whose name satisfies ``pred`` (e.g. MoE routers
        under ``freeze_moe_router``): their gradients are zeroed after the
        data-parallel reduction (they count neither in the clip norm nor in the
        moments) and they take no weight decay, so AdamW leaves them unchanged.
        Returns the number of frozen elements in this rank's shards."""
        n = 0
        for seg in self.segments:
            fr = []
            for sp, _ in self.model.named_flat_params():
                if not pred(sp.name):
                    continue
                a, b = max(sp.offset, seg.s_lo), min(sp.offset + sp.numel, seg.s_hi)
                if a < b:
                    fr.append((a - seg.s_lo, b - seg.s_lo, False))
            if not fr:
                continue
            seg.frozen_ranges = [(a, b) for a, b, _ in _merge(fr)]
            n += sum(b - a for a, b in seg.frozen_ranges)
            # split the decay ranges so the frozen ones take no decay
            cuts = sorted({x for a, b in seg.frozen_ranges for x in (a, b)})
            out = []
            for a, b, d in seg.wd_ranges:
                pts = [a] + [c for c in cuts if a < c < b] + [b]
                for lo, hi in zip(pts[:-1], pts[1:]):
                    frozen = any(fa <= lo and hi <= fb for fa, fb in seg.frozen_ranges)
                    out.append((lo, hi, d and not frozen))
            seg.wd_ranges = _merge(out)
            nd = [(a, b) for a, b, d in seg.wd_ranges if not d]
            seg.nodecay_dev = torch.tensor(nd if nd else [[seg.shard, seg.shard]], dtype=torch.int64,
                                           device=self.device).view(-1, 2)
        return n

    # ------------------------------------ reduction overlapped with backward
    def setup_overlap(self, layer_of) -> bool:
        """Megatron's ``overlap_grad_reduce`` for the fused data-parallel path.

        The dense segment's parameters are bucketed by decoder layer
        (``layer_of(name)`` -> layer index or None).  During the backward pass of
        a step's last micro-batch, when a layer's gradients are final
        (``layer_ready``, called from an autograd hook on the layer's input), each
        rank publishes the step's epoch for that layer in a symmetric word array
        (stream memory write on the compute stream), and a side stream waits until
        every DP rank published it (bounded wait kernel) and reduces this rank's
        part of the layer's range out of the peers' gradient buffers (the same
        peer-load reduction as ``step``).  ``step`` then reduces only what no
        bucket covered (embedding, final norm, head, parameters that are first
        summed over TP).  Collective (allocates symmetric memory); returns whether
        overlap is on (the fused DP path only, no pipeline parallelism)."""
        seg = self.segments[0]
        if not self._fused(seg) or self.pp_group is not None:
            return False
        ranges: dict[int, list] = {}
        params: dict[int, list] = {}
        for sp, p in self.model.named_flat_params():
            L = layer_of(sp.name)
            if L is None or sp.ep_dim is not None or not (seg.lo <= sp.offset < seg.hi):
                continue
            mode = getattr(sp, "grad_reduce", None)
            if self.tp > 1 and (mode == "tp_sum" or (mode is None and self.sequence_parallel and sp.tp_dim is None)):
                continue  # summed over TP in step() before the data-parallel reduction
            end = min(seg.hi, sp.offset + (sp.numel + 63) // 64 * 64)  # through the parameter's padding
            ranges.setdefault(L, []).append((sp.offset, end, True))
            params.setdefault(L, []).append(p)
        mine = {}
        for L, rs in ranges.items():
            cut = [(max(a, seg.s_lo), min(b, seg.s_hi)) for a, b, _ in _merge(rs)]
            mine[L] = [(a, b) for a, b in cut if a < b]
        n_layers = int(self.model.cfg.num_layers)
        flags = self.symmetric.alloc(4 * n_layers)
        flags.local_view(torch.int32, n_layers).zero_()
        torch.cuda.synchronize()
        self._fence(seg.group)
        self._ov = {"mine": mine, "params": params, "flags": flags, "epoch": 0,
                    "flag_ptrs": [flags.ptrs[dist.get_global_rank(seg.group, r)] for r in range(seg.n)],
                    "stream": torch.cuda.Stream(device=self.device), "parts": [], "done": set()}
        return True

    def begin_overlap(self) -> bool:
        """Arm the overlapped reduction for the backward pass that follows (the
        step's last micro-batch).  The ranks first meet (a fence on the compute
        stream), so the readiness waits only absorb the skew of one backward."""
        ov = self._ov
        if ov is None:
            return False
        self.ensure_grad_buffer()
        seg = self.segments[0]
        self._fence(seg.group)
        ov["epoch"] += 1
        ov["parts"], ov["done"] = [], set()
        ov["stream"].wait_stream(torch.cuda.current_stream())
        self._ov_active = True
        return True

    def layer_ready(self, layer: int) -> None:
        """Layer ``layer``'s gradients are complete on this rank (autograd hook)."""
        ov = self._ov
        if not self._ov_active or ov is None or layer not in ov["params"] or layer in ov["done"]:
            return
        for p in ov["params"][layer]:  # gradients autograd left in .grad (router weights)
            if p.grad is not None:
                p.main_grad.add_(p.grad.float())
                p.grad = None
        e = ext()
        flags = ov["flags"]
        e.stream_write_u32(flags.local_ptr + 4 * layer, ov["epoch"])
        ready = torch.cuda.Event()
        ready.record()
        seg = self.segments[0]
        side = ov["stream"]
        with torch.cuda.stream(side):
            side.wait_event(ready)
            e.dp_wait_ready(ov["flag_ptrs"], layer, ov["epoch"])
            ptrs = self._peer_ptrs(self._grad_symm, seg)
            for a, b in ov["mine"].get(layer, []):
                ov["parts"].append(e.dp_reduce_shard(ptrs, a, b - a, seg.grad_shard[a - seg.s_lo:b - seg.s_lo]))
        ov["done"].add(layer)

    def _overlap_rest(self, seg) -> list:
        """Ranges of this rank's shard that no completed bucket reduced."""
        covered = sorted(r for L in self._ov["done"] for r in self._ov["mine"].get(L, []))
        rest, cur = [], seg.s_lo
        for a, b in covered:
            if a > cur:
                rest.append((cur, a))
            cur = max(cur, b)
        if cur < seg.s_hi:
            rest.append((cur, seg.s_hi))
        return rest

    # ----------------------------------------------------------------- step
    @torch.no_grad()
    def step(self) -> dict:
        self.ensure_grad_buffer()
        self._fold_param_grads()
        overlapped = self._ov_active
        if overlapped:
            # the buckets reduced during the backward are complete before they are read
            torch.cuda.current_stream().wait_stream(self._ov["stream"])
            self._ov_active = False
        m = self.model
        if self.tp > 1:
            for sp, p in m.named_flat_params():
                mode = getattr(sp, "grad_reduce", None)
                # replicated params saw different tokens on each TP rank under SP;
                # some (LoRA A of column-parallel layers) hold partial sums always
                if mode == "tp_sum" or (mode is None and self.sequence_parallel and sp.tp_dim is None
                                        and sp.ep_dim is None):
                    dist.all_reduce(p.main_grad, group=self.tp_group)
        sq_total = torch.zeros((), dtype=torch.float32, device=self.device)
        for seg in self.segments:
            fused = self._fused(seg)
            if not seg.sharded and seg.n > 1:
                dist.all_reduce(seg.grad_shard, group=seg.group)  # replicated (Muon): whole gradient
            if seg.sharded and fused:
                # peers finished their backward passes (stream-ordered fence), then
                # this rank reduces its shard straight out of their gradient buffers
                self._fence(seg.group)
                ptrs = self._peer_ptrs(self._grad_symm, seg)
                if overlapped and seg is self.segments[0]:
                    parts = list(self._ov["parts"])
                    for a, b in self._overlap_rest(seg):
                        parts.append(ext().dp_reduce_shard(ptrs, a, b - a, seg.grad_shard[a - seg.s_lo:b - seg.s_lo]))
                    sq_all = torch.cat([p.reshape(-1) for p in parts]).sum()
                    self._ov["parts"] = []
                else:
                    part = ext().dp_reduce_shard(ptrs, seg.s_lo, seg.shard, seg.grad_shard)
                    sq_all = part.sum()
            elif seg.sharded:
                # losses are normalised by GLOBAL token / sequence counts, so the
                # per-rank gradients are partial sums: reduce with SUM, not mean.
                dist.reduce_scatter_tensor(seg.grad_shard, self.main_grad[seg.lo:seg.hi], group=seg.group)
            g = seg.grad_shard
            if seg.frozen_ranges:
                for a, b in seg.frozen_ranges:
                    g[a:b].zero_()
                if seg.sharded and fused:
                    sq_all = sum_of_squares(g)  # the fused partials included the frozen gradients
            if not (seg.sharded and fused):
                sq_all = sum_of_squares(g)
            if self.tp > 1:
                sq_rep = torch.zeros((), dtype=torch.float32, device=g.device)
                for a, b in seg.rep_ranges:
                    sq_rep = sq_rep + sum_of_squares(g[a:b])
                sq_sh = sq_all - sq_rep
                dist.all_reduce(sq_sh, group=self.tp_group)
                sq = sq_sh + sq_rep
            else:
                sq = sq_all
            if seg.sharded:
                dist.all_reduce(sq, group=seg.group)
            if seg.norm_sum_group is not None and _ws(seg.norm_sum_group) > 1:
                dist.all_reduce(sq, group=seg.norm_sum_group)
            sq_total = sq_total + sq
        if self.pp_group is not None:
            dist.all_reduce(sq_total, group=self.pp_group)
        norm = float(sq_total.sqrt())
        self.last_grad_norm = norm
        scale = 1.0
        if self.max_grad_norm and self.max_grad_norm > 0 and norm > self.max_grad_norm:
            scale = self.max_grad_norm / (norm + 1e-6)
        if not math.isfinite(norm):
            self.zero_grad()
            return {"grad_norm": norm, "lr": self.current_lr(), "skipped": 1.0}
        self.step_count += 1
        lr = self.scheduler.lr_at(self.step_count - 1)
        fenced = False
        for seg in self.segments:
            out = m.flat_param[seg.s_lo:seg.s_hi]
            g = seg.grad_shard
            if seg.sharded and self._fused(seg):
                ext().dp_adam_allgather(self._peer_ptrs(self._flat_symm(), seg, param=True), seg.s_lo, seg.master, g,
                                        seg.exp_avg, seg.exp_avg_sq, seg.nodecay_dev, lr, self.beta1, self.beta2,
                                        self.eps, self.weight_decay, self.step_count, scale)
                fenced = True
                continue
            for a, b, decayed in seg.wd_ranges:
                adamw_step(seg.master[a:b], g[a:b], seg.exp_avg[a:b], seg.exp_avg_sq[a:b], lr, self.beta1,
                           self.beta2, self.eps, self.weight_decay if decayed else 0.0, self.step_count,
                           grad_scale=scale, param_out=out[a:b])
            if seg.muon_params:
                self._muon_step(seg, out, lr, scale)
            if seg.sharded:
                dist.all_gather_into_tensor(m.flat_param[seg.lo:seg.hi], out.clone(), group=seg.group)
        if fenced:
            # every rank's peer stores of its updated shard must land before the
            # parameters are read (or the gradients zeroed under a peer's loads)
            for seg in self.segments:
                if seg.sharded and self._fused(seg):
                    self._fence(seg.group)
        self.zero_grad()
        bump = getattr(m, "bump_weight_version", None)
        if bump is not None:
            bump()
        return {"grad_norm": norm, "lr": lr}

    # ------------------------------------------------------ fused DP path
    def _muon_step(self, seg, out: torch.Tensor, lr: float, grad_scale: float) -> None:
        from rl_b200.parallel.muon import muon_scale, orthogonalize

        cfg = self.muon
        mu = cfg.momentum
        for sp, a, b in seg.muon_params:
            if any(fa <= a and b <= fb for fa, fb in seg.frozen_ranges):
                continue  # frozen (e.g. MoE router): no update
            shape = sp.shape
            g = seg.grad_shard[a:b].view(shape) * grad_scale
            buf = seg.exp_avg[a:b].view(shape)
            buf.lerp_(g, 1.0 - mu)
            upd = g.lerp(buf, mu) if cfg.nesterov else buf
            tp_dim = None if sp.tp_dim is None else sp.tp_dim - len(shape)  # counted from the end
            blocks = [upd]
            if cfg.split_qkv and sp.name.endswith("qkv_proj.weight"):
                hd = self.model.cfg.head_dim
                blocks = list(torch.split(upd, [self.model.nq * hd, self.model.nkv * hd, self.model.nkv * hd], -2))
            outs = []
            for blk in blocks:
                o, (d_out, d_in) = orthogonalize(blk, tp_dim, cfg, self.tp_group)
                outs.append(o * (muon_scale(d_out, d_in, cfg.scale_mode) * cfg.extra_scale_factor))
            o = torch.cat(outs, -2) if len(outs) > 1 else outs[0]
            w = seg.master[a:b].view(shape)
            if self.weight_decay and not sp.no_weight_decay:
                w.mul_(1.0 - lr * self.weight_decay)
            w.add_(o, alpha=-lr)
            out[a:b].copy_(w.reshape(-1))

    def _fused(self, seg) -> bool:
        if not seg.sharded:
            return False
        return (self.symmetric is not None and not seg.expert and self.device.type == "cuda"
                and self._flat_symm() is not None)

    def _flat_symm(self):
        return getattr(self.model.flat_param, "_symm", None)

    def _fence(self, group) -> None:
        x = torch.zeros(1, device=self.device)
        dist.all_reduce(x, group=group)

    def _peer_ptrs(self, buf, seg, param: bool = False) -> list[int]:
        """Base addresses of every group rank's buffer (group-rank order) on this GPU."""
        key = ("p" if param else "g", id(buf), id(seg.group))
        cache = self.__dict__.setdefault("_ptr_cache", {})
        if key not in cache:
            cache[key] = [buf.ptrs[dist.get_global_rank(seg.group, r)] for r in range(seg.n)]
        return cache[key]

    def current_lr(self) -> float:
        return self.scheduler.lr_at(max(0, self.step_count - 1))

    @torch.no_grad()
    def restore_params_from_master(self) -> None:
        """Rewrite the bf16 parameters from the fp32 master shards (after a weight swap)."""
        m = self.model
        if getattr(m, "bump_weight_version", None) is not None:
            m.bump_weight_version()
        for seg in self.segments:
            m.flat_param[seg.s_lo:seg.s_hi].copy_(seg.master)
            if seg.sharded:
                dist.all_gather_into_tensor(m.flat_param[seg.lo:seg.hi], m.flat_param[seg.s_lo:seg.s_hi].clone(),
                                            group=seg.group)

    # ---------------------------------------------------------- state dict
    def state_dict(self) -> dict:
        return {"segments": [{"master": s.master.cpu(), "exp_avg": s.exp_avg.cpu(), "exp_avg_sq": s.exp_avg_sq.cpu(),
                              "s_lo": s.s_lo, "s_hi": s.s_hi} for s in self.segments],
                "step": self.step_count, "padded": self.padded}

    def load_state_dict(self, sd: dict) -> None:
        segs = sd["segments"]
        if len(segs) != len(self.segments) or any(a["s_lo"] != b.s_lo or a["s_hi"] != b.s_hi
                                                   for a, b in zip(segs, self.segments)):
            raise ValueError("optimizer shard layout mismatch (different parallel layout?)")
        for a, b in zip(segs, self.segments):
            b.master.copy_(a["master"])
            b.exp_avg.copy_(a["exp_avg"])
            b.exp_avg_sq.copy_(a["exp_avg_sq"])
        self.step_count = int(sd["step"])
        self.restore_params_from_master()

    def offload(self) -> None:
        for seg in self.segments:
            for name in ("master", "exp_avg", "exp_avg_sq"):
                t = getattr(seg, name)
                if t.is_cuda:
                    setattr(seg, name, t.cpu())

    def onload(self, device) -> None:
        for seg in self.segments:
            for name in ("master", "exp_avg", "exp_avg_sq"):
                t = getattr(seg, name)
                if not t.is_cuda:
                    setattr(seg, name, t.to(device))
