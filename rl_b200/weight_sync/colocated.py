"""Colocated refit transports (trainer and rollout engine share each GPU)."""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from rl_b200.weight_sync.interfaces import WeightSynchronizer
from rl_b200.weight_sync.reshard import (apply_regions_reference, build_regions, copy_tasks, quant_layout,
                                         quant_regions_reference, quant_tasks)

__all__ = ["ColocatedInPlaceSynchronizer", "ColocatedReshardSynchronizer", "LoRAMergeSynchronizer",
           "PipelineGatherSynchronizer"]


class LoRAMergeSynchronizer:
    """LoRA training: the rollout copy holds base + scale * B A (merged once per
    refit, so decode runs plain GEMMs)."""
    name = "lora_merge"

    def __init__(self, lora, gen_model):
        self.lora, self.gen_model = lora, gen_model
        self.version = 0

    def sync(self) -> dict:
        self.lora.merged_into(self.gen_model)
        self.version += 1
        return {"version": self.version}

    def shutdown(self) -> None:
        pass


class ColocatedInPlaceSynchronizer(WeightSynchronizer):
    """Same layout: the optimizer step already wrote the bf16 weights the
    engine reads (the flat parameter buffer is shared), nothing to move."""
    name = "inplace"

    def _sync(self) -> int:
        return 0


class ColocatedReshardSynchronizer(WeightSynchronizer):
    """Training TP ``t`` -> generation TP ``g`` (``g`` divides ``t``), optionally
    quantising the linear weights to 128x128 block-scaled e4m3.

    On CUDA the training flat buffers are symmetric memory (``peer_ptrs[r]`` is
    TP rank r's buffer mapped on this GPU) and ONE native launch per output
    kind does the whole reshard (``rl_b200._C.refit_copy`` / ``refit_quant_fp8``).
    On CPU (gloo tests) the shards are all-gathered and the same region table is
    applied with torch indexing."""
    name = "reshard"

    def __init__(self, train_model, gen_model, tp_group, tp_rank: int, tp_size: int,
                 peer_ptrs: Optional[list[int]] = None, fp8: bool = False, pow2_scales: bool = False,
                 copy_bf16: bool = True):
        super().__init__()
        self.train_model, self.gen_model = train_model, gen_model
        self.group, self.rank, self.t = tp_group, tp_rank, tp_size
        self.g = gen_model.ps.tp_size
        self.peer_ptrs = peer_ptrs
        self.fp8, self.pow2, self.copy_bf16 = fp8, pow2_scales, copy_bf16
        self.regions = build_regions(train_model.specs, gen_model.specs, train_model.cfg, self.t, self.g, tp_rank)
        self.dev = gen_model.flat_param.device
        self.native = self.dev.type == "cuda"
        self.q_layout, qbytes, nscales = quant_layout(gen_model.specs) if fp8 else ({}, 0, 0)
        self.q = torch.zeros(qbytes, dtype=torch.uint8, device=self.dev) if fp8 else None
        self.scales = torch.zeros(nscales, dtype=torch.float32, device=self.dev) if fp8 else None
        self._tasks = self._qtasks = None
        if self.native:
            if peer_ptrs is None or len(peer_ptrs) != self.t:
                raise ValueError("native reshard needs the TP peers' symmetric parameter buffers")
            if copy_bf16:
                self._tasks = torch.from_numpy(copy_tasks(self.regions, peer_ptrs)).to(self.dev)
            if fp8:
                self._qtasks = torch.from_numpy(quant_tasks(self.regions, self.q_layout, peer_ptrs)).to(self.dev)

    def fp8_weight(self, name: str):
        """(e4m3 ``[R, C]``, fp32 scales ``[ceil(R/128), ceil(C/128)]``) views of one quantised weight."""
        qoff, soff, R, C, nb, kb = self.q_layout[name]
        return (self.q[qoff: qoff + R * C].view(torch.float8_e4m3fn).view(R, C),
                self.scales[soff: soff + nb * kb].view(nb, kb))

    def _fence(self) -> None:
        # every TP peer's optimizer step must be complete before its shard is read:
        # a stream-ordered all-reduce on the TP group orders this rank's kernels
        # after the peers' preceding work
        if self.t > 1:
            x = torch.zeros(1, device=self.dev)
            dist.all_reduce(x, group=self.group)

    def _sync(self) -> int:
        nbytes = 0
        if self.native:
            from rl_b200.ops._ext import ext

            self._fence()
            if self._tasks is not None:
                ext().refit_copy(self._tasks, self.gen_model.flat_param)
                nbytes += self.gen_model.flat_param.numel() * 2
            if self._qtasks is not None:
                ext().refit_quant_fp8(self._qtasks, self.q, self.scales, self.pow2)
                nbytes += self.q.numel() + self.scales.numel() * 4
            # peers must finish reading this rank's shard before its next optimizer
            # step overwrites it; their next TP collective (in the next training
            # step, after this kernel in their stream order) gives that order
            return nbytes
        src = self.train_model.flat_param.detach()
        if self.t > 1:
            shards = [torch.empty_like(src) for _ in range(self.t)]
            dist.all_gather(shards, src.contiguous(), group=self.group)
        else:
            shards = [src]
        with torch.no_grad():
            apply_regions_reference(self.regions, shards, self.gen_model.flat_param)
            if self.fp8:
                quant_regions_reference(self.gen_model.flat_param, self.q_layout, self.q, self.scales,
                                        self.gen_model.specs, self.pow2)
        return self.gen_model.flat_param.numel() * self.gen_model.flat_param.element_size()


def regions_bytes(regions) -> int:
    return int(np.sum([r.rows * r.cols for r in regions])) * 2


class PipelineGatherSynchronizer(WeightSynchronizer):
    """Pipeline-parallel training -> full-depth rollout copy on every stage.

    Each stage's flat parameter buffer is broadcast over the pipeline group in
    one collective (NVLink, no host hop); every rank then copies the named
    slices into its rollout model.  The per-stage layouts (name, offset, numel)
    are exchanged once at construction.  The rollout copy keeps the training
    TP layout, so only depth is gathered."""
    name = "pp_gather"

    def __init__(self, train_model, gen_model, pp_group, pp_ranks: list, stage: int):
        super().__init__()
        self.train_model, self.gen_model = train_model, gen_model
        self.group, self.ranks, self.stage = pp_group, list(pp_ranks), stage
        mine = ([(sp.name, sp.offset, sp.numel) for sp in train_model.specs], int(train_model.flat_param.numel()))
        self.layouts: list = [None] * len(self.ranks)
        dist.all_gather_object(self.layouts, mine, group=pp_group)
        names = {n for lay, _ in self.layouts for n, _, _ in lay}
        missing = [sp.name for sp in gen_model.specs if sp.name not in names]
        if missing:
            raise ValueError(f"rollout parameters held by no pipeline stage: {missing[:4]}")

    @torch.no_grad()
    def _sync(self) -> int:
        flat = self.train_model.flat_param
        nbytes = 0
        stage_buf = None
        gen = self.gen_model._params
        for s, (lay, n) in enumerate(self.layouts):
            if s == self.stage:
                buf = flat
            else:
                if stage_buf is None or stage_buf.numel() < n:
                    stage_buf = torch.empty(max(n for _, n in self.layouts), dtype=flat.dtype, device=flat.device)
                buf = stage_buf[:n]
            dist.broadcast(buf, src=self.ranks[s], group=self.group)
            for name, off, numel in lay:
                if name in gen:
                    gen[name].data.view(-1).copy_(buf[off:off + numel])
                    nbytes += numel * buf.element_size()
        return nbytes


class NVFP4RolloutSynchronizer(WeightSynchronizer):
    """Rollout weights in NVFP4 (``generation.vllm_cfg.precision: nvfp4``): the
    trained bf16 buffer is copied into the rollout model's own buffer and every
    linear-layer weight (not the embeddings, LM head, norms or MoE routers, the
    reference's default NVFP4 ignore list) is replaced by its NVFP4 round trip
    (``quant_nvfp4``: e2m1 codes, e4m3 16-element block scales, fp32 tensor scale).
    The rollout therefore samples from the NVFP4-weight model (W4A16: the GEMMs
    run in bf16 on the dequantised values); ``stats["nvfp4_bytes"]`` is the packed
    size of the quantised weights.

    Reference: NVFP4 rollout quantisation
    (``nemo_rl/models/generation/vllm/quantization/nvfp4_pertoken.py``) and the
    ModelOpt real-quant rollout."""
    name = "nvfp4"

    def __init__(self, model, gen_model):
        super().__init__()
        self.model, self.gen_model = model, gen_model

    @staticmethod
    def quantized(name: str) -> bool:
        if not name.endswith("weight") and not name.endswith(("gate_up_proj", "down_proj")):
            return False
        return any(k in name for k in ("self_attn.", "mlp.")) and not name.endswith("mlp.gate.weight") \
            and "norm" not in name

    @torch.no_grad()
    def _sync(self) -> int:
        from rl_b200.models.quantization import dequant_nvfp4, quant_nvfp4

        # by name: the optimizer may have re-laid the trained buffer out (padding, expert shift)
        src = {sp.name: q for sp, q in self.model.named_flat_params()}
        packed = 0
        for sp, p in self.gen_model.named_flat_params():
            w = src[sp.name]
            if not self.quantized(sp.name):
                p.copy_(w)
                continue
            t = quant_nvfp4(w.reshape(-1, w.shape[-1]))  # experts' [E, rows, cols] stacks quantise row by row
            p.copy_(dequant_nvfp4(t, p.dtype).view(p.shape))
            packed += t.nbytes
        bump = getattr(self.gen_model, "bump_weight_version", None)
        if bump is not None:
            bump()
        self.stats["nvfp4_bytes"] = packed
        return self.model.flat_param.numel() * self.model.flat_param.element_size()
