"""Per-GPU policy worker: trainer + rollout engine + reference policy on one device.

Implements the policy-worker surface of the reference
(``MegatronPolicyWorkerImpl`` ``nemo_rl/models/policy/workers/megatron_policy_worker.py:693``:
``train`` ``:1382``, ``get_logprobs`` ``:2643``, ``use_reference_model`` ``:3128``,
``offload_before_refit`` ``:4853``, ``save_checkpoint`` ``:5017``) for the SPMD
design of this framework: every rank runs one worker; data arrive already
sharded by data-parallel rank, and tensor-parallel peers see identical data.

Training step (per global batch):
  pack rows into token-budgeted micro-batches (sequence packing) ->
  packed forward (THD) -> fused LM-head+logprob -> loss on padded [B, S-1]
  views -> backward into fp32 main-grad buffers -> distributed AdamW step.
"""

from __future__ import annotations

import contextlib
import math
import os
import time
from typing import Any, Optional

import numpy as np
import torch
import torch.distributed as dist

from rl_b200.data.packing import get_packer
from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.models.config import ModelConfig, apply_hf_config_overrides, get_model_config
from rl_b200.parallel.muon import MuonConfig
from rl_b200.models.generation.engine import RolloutEngine
from rl_b200.models.transformer import TransformerLM
from rl_b200.ops.fused_linear_logprob import linear_logprobs
from rl_b200.parallel.dist_optimizer import FlatAdamW
from rl_b200.parallel.state import ParallelState, get_parallel_state
from rl_b200.utils.timer import Timer

__all__ = ["PolicyWorker", "TrainStepState", "pack_rows"]


class TrainStepState:
    """State of one optimizer step between ``begin_train_step`` and
    ``finish_train_step`` (micro-batch plan, device batch, global counts)."""

    def __init__(self, **kw):
        self.__dict__.update(kw)
        self.mb_metrics: list[dict] = []
        self.done = 0

    @property
    def num_microbatches(self) -> int:
        return len(self.plan)


def _dtype(precision: str) -> torch.dtype:
    return {"bfloat16": torch.bfloat16, "bf16": torch.bfloat16, "float32": torch.float32, "fp32": torch.float32,
            "float16": torch.float16}.get(str(precision), torch.bfloat16)


def _to_device(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """Host tensor -> device via pinned memory (asynchronous on the current stream)."""
    if dev.type != "cuda" or t.is_cuda:
        return t.to(dev)
    return t.pin_memory().to(dev, non_blocking=True)


def pack_rows(input_ids: torch.Tensor, lengths: list[int], rows: list[int], pad_to_multiple: int = 1):
    """Concatenate the unpadded rows into one packed sequence batch.

    Returns (flat_ids [T], positions [T] int32, cu_seqlens [n+1] int32, max_len,
    T_real).  When ``pad_to_multiple`` > 1 a dummy tail sequence pads T up to the
    multiple (needed for sequence parallelism)."""
    pieces, pos, cu = [], [], [0]
    for r in rows:
        L = int(lengths[r])
        pieces.append(input_ids[r, :L])
        pos.append(torch.arange(L, dtype=torch.int32))
        cu.append(cu[-1] + L)
    T = cu[-1]
    pad = (-T) % pad_to_multiple
    if pad:
        pieces.append(torch.zeros(pad, dtype=input_ids.dtype))
        pos.append(torch.arange(pad, dtype=torch.int32))
        cu.append(cu[-1] + pad)
    flat = torch.cat(pieces) if pieces else torch.zeros(0, dtype=input_ids.dtype)
    max_len = max((cu[i + 1] - cu[i]) for i in range(len(cu) - 1)) if len(cu) > 1 else 0
    return flat, torch.cat(pos), torch.tensor(cu, dtype=torch.int32), max_len, T


class PolicyWorker:
    def __init__(self, policy_cfg: dict, model_cfg: Optional[ModelConfig] = None,
                 pstate: Optional[ParallelState] = None, seed: int = 0, init_reference_model: bool = True,
                 loss_cfg: Optional[dict] = None):
        self.cfg = policy_cfg
        self.ps = pstate or get_parallel_state()
        self.device = self.ps.device
        self.model_cfg = apply_hf_config_overrides(
            model_cfg or get_model_config(policy_cfg.get("model_name", "tiny-llama")),
            policy_cfg.get("hf_config_overrides"), policy_cfg.get("max_total_sequence_length"))
        self.dtype = _dtype(policy_cfg.get("precision", "bfloat16"))
        if self.device.type == "cpu" and self.dtype != torch.float32:
            self.dtype = torch.float32
        mc = policy_cfg.get("megatron_cfg", {}) or {}
        uneven = {k: int(mc[k]) for k in ("num_layers_in_first_pipeline_stage", "num_layers_in_last_pipeline_stage",
                                          "virtual_pipeline_model_parallel_size") if mc.get(k) is not None}
        if uneven:
            self.model_cfg = self.model_cfg.replace(extra={**self.model_cfg.extra, **uneven})
        self.sequence_parallel = bool(mc.get("sequence_parallel", False)) and self.ps.tp_size > 1
        act_ckpt = bool(mc.get("activation_checkpointing", policy_cfg.get("activation_checkpointing", False)))
        self.num_labels = int(policy_cfg.get("num_labels", 0) or 0)  # > 0: value / reward model
        gen_cfg = dict(policy_cfg.get("generation", {}) or {})
        vcfg = gen_cfg.get("vllm_cfg", {}) or {}
        # rollout tensor parallelism: the training TP size (same layout, in-place refit)
        # or 1 (every GPU holds full rollout weights; refit reshards over NVLink)
        self.gen_tp = int(gen_cfg.get("tensor_parallel_size") or vcfg.get("tensor_parallel_size")
                          or self.ps.tp_size)
        if self.gen_tp not in (1, self.ps.tp_size):
            raise NotImplementedError(f"generation TP {self.gen_tp} must be 1 or the training TP {self.ps.tp_size}")
        self.fp8_rollout = str(vcfg.get("precision", gen_cfg.get("precision", "bfloat16"))).lower() == "fp8"
        self.nvfp4_rollout = str(vcfg.get("precision", gen_cfg.get("precision", "bfloat16"))).lower() == "nvfp4"
        # fp8 rollout scales: powers of two (hardware-scaled GEMM) unless a config
        # turns the reference's pow2 options off (then fp32 scales, promoting GEMM)
        self.fp8_pow2 = vcfg.get("pow2_weight_scaling_factors") is not False and \
            vcfg.get("pow2_activation_scaling_factors") is not False
        resharded = self.gen_tp != self.ps.tp_size
        self.pp = self.ps.pp_size
        if self.pp > 1:
            for what, bad in (("context parallelism", self.ps.cp_size > 1), ("a different rollout TP", resharded),
                              ("LoRA", bool((policy_cfg.get("lora_cfg") or mc.get("lora_cfg") or {}).get("enabled"))),
                              ("fp8 rollout weights", self.fp8_rollout)):
                if bad:
                    raise NotImplementedError(f"pipeline parallelism with {what}")
        # symmetric memory (every rank of the node maps every other's parameter and
        # gradient buffers): needed by the reshard refit and the fused DP optimizer
        from rl_b200.parallel.symm import NodeSymmetric

        fused_dp = bool(mc.get("fused_dp_optimizer", True)) and self.ps.dp_size > 1
        self.symmetric = NodeSymmetric() if NodeSymmetric.supported() and (
            (resharded and self.ps.tp_size > 1) or fused_dp) else None
        flat_alloc = self.symmetric.flat_alloc if self.symmetric is not None else None
        self.model = TransformerLM(self.model_cfg, self.ps, device=self.device, dtype=self.dtype, seed=seed,
                                   sequence_parallel=self.sequence_parallel, activation_checkpointing=act_ckpt,
                                   num_labels=self.num_labels, flat_alloc=flat_alloc,
                                   expert_tensor_parallel=mc.get("expert_tensor_parallel_size"))
        etp = self.model.etp
        f8 = mc.get("fp8_cfg") or {}
        if f8.get("enabled", False):
            if str(f8.get("fp8", "e4m3")).lower() != "e4m3" or \
                    str(f8.get("fp8_recipe", "blockwise")).lower() not in ("blockwise", "mxfp8"):
                raise NotImplementedError(f"fp8 training recipe {f8.get('fp8')}/{f8.get('fp8_recipe')}")
            # power-of-two (E8M0) block scales unless turned off: the tensor cores apply them
            self.model.fp8_train = {"pow2": bool(f8.get("pow2_scales", True))}
        from rl_b200.models.quantization import QAT, QATConfig

        qcfg = QATConfig.from_cfg(policy_cfg.get("quant_cfg"))
        if qcfg is not None:
            if self.model.fp8_train is not None:
                raise ValueError("quant_cfg (fake-quantised training) and fp8_cfg (fp8 GEMMs) are exclusive")
            self.model.qat = QAT(qcfg)
        from rl_b200.models.lora import LoRAAdapters, LoRAConfig

        lcfg = LoRAConfig(policy_cfg.get("lora_cfg") or mc.get("lora_cfg")
                          or (policy_cfg.get("dtensor_cfg") or {}).get("lora_cfg"))
        self.lora = None
        opt_target = self.model
        if lcfg.enabled:
            # base weights frozen; the optimizer steps the adapters' flat buffer
            for prm in self.model._params.values():
                prm.requires_grad_(False)
            self.lora = LoRAAdapters(self.model, lcfg, seed=seed)
            self.model.lora = self.lora
            opt_target = self.lora
            fused_dp = False
            if lcfg.restore_from:
                self.lora.load_peft(lcfg.restore_from)
        opt = policy_cfg.get("optimizer", {}) or {}
        kw = dict(opt.get("kwargs", {}) or {})
        mopt = mc.get("optimizer", {}) or {}
        lr = float(kw.get("lr", mopt.get("lr", 1e-5)))
        betas = kw.get("betas", [mopt.get("adam_beta1", 0.9), mopt.get("adam_beta2", 0.999)])
        eps = float(kw.get("eps", mopt.get("adam_eps", 1e-8)))
        wd = float(kw.get("weight_decay", mopt.get("weight_decay", 0.0)))
        sched = policy_cfg.get("scheduler") if policy_cfg.get("scheduler") is not None else mc.get("scheduler")
        grad_group = self.ps.dp_cp_group if self.ps.cp_size > 1 else self.ps.dp_group
        self.optimizer = FlatAdamW(opt_target, lr=lr, betas=tuple(float(b) for b in betas), eps=eps, weight_decay=wd,
                                   max_grad_norm=policy_cfg.get("max_grad_norm", 1.0), scheduler_cfg=sched,
                                   min_lr=float(mopt.get("min_lr", 0.0)), dp_group=grad_group,
                                   tp_group=self.ps.tp_group, sequence_parallel=self.sequence_parallel,
                                   edp_group=self.ps.edp_group, ep_group=self.ps.ep_group,
                                   symmetric=self.symmetric if fused_dp else None,
                                   pp_group=self.ps.pp_group if self.pp > 1 else None,
                                   muon=MuonConfig.from_megatron(mopt) if self.lora is None else None)
        if mc.get("freeze_moe_router", False) and self.model_cfg.is_moe:
            # the reference's GRPO default: routers keep their initial weights
            self.optimizer.freeze(lambda name: name.endswith("mlp.gate.weight"))
        # overlap_grad_reduce: data-parallel gradient reduction per decoder layer during
        # the backward of a step's last micro-batch (fused DP path)
        ddp = mc.get("distributed_data_parallel_config") or {}
        self._overlap_grad_reduce = bool(ddp.get("overlap_grad_reduce", False)) and self.optimizer.setup_overlap(
            lambda name: int(name.split(".")[2]) if name.startswith("model.layers.") else None)
        mgc = gen_cfg.get("mcore_generation_config", {}) or {}
        self.max_seq_len = int(policy_cfg.get("max_total_sequence_length", 512))
        if self.max_seq_len > self.model.rope_cache.shape[0]:
            raise ValueError(f"max_total_sequence_length {self.max_seq_len} exceeds the model's "
                             f"{self.model.rope_cache.shape[0]} rotary positions; raise max_position_embeddings "
                             "(policy.hf_config_overrides) or extend the context with YaRN rope_scaling")
        self.gen_model = self.model
        if self.lora is not None:
            # rollout copy with the adapters merged in (same TP layout)
            self.gen_model = TransformerLM(self.model_cfg, self.ps, device=self.device, dtype=self.dtype,
                                           skip_init=True, expert_tensor_parallel=etp)
        elif self.pp > 1:
            # rollout runs the whole depth on every stage's GPU (same TP layout);
            # the refit gathers the other stages' layers over the pipeline group
            import dataclasses

            gps = dataclasses.replace(self.ps, pp_size=1, pp_rank=0, pp_group=None, pp_ranks=[self.ps.rank])
            self.gen_model = TransformerLM(self.model_cfg, gps, device=self.device, dtype=self.dtype,
                                           skip_init=True, expert_tensor_parallel=etp)
        elif self.nvfp4_rollout:
            if resharded:
                raise NotImplementedError("NVFP4 rollout weights with a different rollout TP")
            # rollout copy holding the NVFP4 round trip of the trained weights (same layout)
            self.gen_model = TransformerLM(self.model_cfg, self.ps, device=self.device, dtype=self.dtype,
                                           skip_init=True, expert_tensor_parallel=etp)
        elif resharded:
            from rl_b200.parallel.state import single_process_state

            self.gen_model = TransformerLM(self.model_cfg, single_process_state(self.device), device=self.device,
                                           dtype=self.dtype, skip_init=True)
        self._expert_bias_rate = 0.0
        if mc.get("moe_router_enable_expert_bias", False) and self.model_cfg.is_moe:
            # aux-loss-free load balancing: the rollout copy must route with the same bias
            if self.gen_model is not self.model:
                raise NotImplementedError("moe_router_enable_expert_bias with a different rollout layout")
            self.model.enable_expert_bias()
            self._expert_bias_rate = float(mc.get("moe_router_bias_update_rate", 1e-3) or 0.0)
        self.weight_sync = self._make_weight_sync(resharded)
        kv_dt = str(vcfg.get("kv_cache_dtype", gen_cfg.get("kv_cache_dtype", "auto"))).lower()
        self._engine_spec = dict(
            max_num_seqs=int(gen_cfg.get("max_num_seqs", 256)),
            kv_dtype=torch.float8_e4m3fn if kv_dt in ("fp8", "fp8_e4m3") else None,
            max_model_len=self.max_seq_len, block_size=int(mgc.get("block_size_tokens", 256)),
            use_cuda_graphs=bool(gen_cfg.get("use_cuda_graphs", True)),
            seed=seed * 7 + self.ps.dp_rank * 100003,
        )
        self._gen_cfg = gen_cfg
        self.engine = RolloutEngine(self.gen_model, gen_cfg, **self._engine_spec)
        # speculative decoding: a small draft LM (same vocab / width, few layers) that
        # proposes tokens for the rollout engine and is trained online on rollouts
        spec = gen_cfg.get("speculative") or {}
        self.draft = None
        self.draft_kind = None
        dpol = policy_cfg.get("draft") or {}
        if dpol.get("enabled", False):
            # Eagle3 head on the policy's hidden states (the reference's policy.draft block);
            # proposals per round from generation.speculative or the vLLM-style speculative_config
            kind = str(dpol.get("speculator_type", "eagle3")).lower()
            if kind not in ("eagle3", "dflash", "mtp"):
                raise NotImplementedError(f"draft speculator_type {kind!r} (eagle3, dflash and mtp are built)")
            from rl_b200.models.eagle3 import DFlashDraft, Eagle3Draft

            sc = ((gen_cfg.get("vllm_kwargs") or {}).get("speculative_config") or {})
            k = int(spec.get("num_speculative_tokens") or sc.get("num_speculative_tokens") or 3)
            if kind == "dflash":  # block drafter: the whole round's proposals in one forward
                self.draft = DFlashDraft(self.gen_model, aux_layers=dpol.get("aux_layers"), seed=seed, block_size=k)
            elif kind == "mtp":
                # multi-token-prediction head: the last layer's hidden state and the next
                # token's embedding through one decoder layer (the Eagle3 head on one feature)
                self.draft = Eagle3Draft(self.gen_model, aux_layers=(self.model_cfg.num_layers - 1,), seed=seed,
                                         ttt_steps=int(dpol.get("ttt_steps", 1)))
                kind = "eagle3"
            else:
                self.draft = Eagle3Draft(self.gen_model, aux_layers=dpol.get("aux_layers"), seed=seed,
                                         ttt_steps=int(dpol.get("ttt_steps", 2)))
            self.draft_kind = kind
            self.draft_loss_weight = float(dpol.get("loss_weight", 1.0))
            self._draft_anchor_cap = int(dpol.get("max_anchors", 2048))  # block drafter: anchors per step
            self._draft_steps = 0
            self._draft_k = k
            self.engine.set_draft(self.draft, k)
            self._draft_opt = torch.optim.AdamW(self.draft.parameters(), lr=float(dpol.get("lr", 1e-4)))
        elif int(spec.get("num_speculative_tokens", 0) or 0) > 0:
            dcfg = self.model_cfg.replace(num_layers=int(spec.get("draft_num_layers", 1)))
            self.draft = TransformerLM(dcfg, self.gen_model.ps, device=self.device, dtype=self.dtype,
                                       seed=seed + 7919)
            self.engine.set_draft(self.draft, int(spec["num_speculative_tokens"]))
            self._draft_opt = torch.optim.AdamW(self.draft.parameters(), lr=float(spec.get("draft_lr", 1e-4)))
        self.ref_flat: Optional[torch.Tensor] = None
        if init_reference_model and self.lora is None:
            self.ref_flat = self.model.flat_param.detach().clone()
        sp = policy_cfg.get("sequence_packing", {}) or {}
        self.train_mb_tokens = int(sp.get("train_mb_tokens", self.max_seq_len * int(policy_cfg.get("train_micro_batch_size", 4))))
        self.logprob_mb_tokens = int(sp.get("logprob_mb_tokens", self.train_mb_tokens))
        self.packing_algorithm = sp.get("algorithm", "modified_first_fit_decreasing")
        # "largest_first" runs the largest packed micro-batch first: the caching
        # allocator's blocks of that one are then reused by every smaller one
        self.microbatch_order = sp.get("microbatch_order") or "packer"
        if self.microbatch_order not in ("packer", "largest_first"):
            raise ValueError(f"sequence_packing.microbatch_order must be 'packer' or 'largest_first', "
                             f"got {self.microbatch_order!r}")
        self.max_sequences_per_bin = sp.get("max_sequences_per_bin")
        self.logprob_chunk = int(policy_cfg.get("logprob_chunk_size") or 4096)
        # colocated rollout needs the HBM of the fp32 gradient buffer for its KV cache
        # HBM plan of the colocated worker: the fp32 gradient buffer (4 bytes/param) is
        # persistent and doubles as the paged KV cache's storage during rollout (the
        # two are never live together); it is re-zeroed at the start of train().
        self.release_grad_after_train = bool(policy_cfg.get("release_grad_after_train", False))
        if bool(policy_cfg.get("kv_cache_in_grad_arena", self.device.type == "cuda")):
            self.engine.kv_arena = lambda: self.optimizer.main_grad
        self.timer = Timer()
        # router replay (R3): the rollout records the experts each MoE layer chose
        # and training / log-prob forwards reuse them
        self.router_replay = bool((policy_cfg.get("router_replay") or {}).get("enabled", False)) \
            and self.model_cfg.is_moe
        if self.router_replay:
            if self.ps.cp_size > 1:
                raise NotImplementedError("router replay with context parallelism")
            self.engine.record_routes = True
        self._routes: Optional[torch.Tensor] = None
        self._pp_comm = None
        self._pp_in: Optional[torch.Tensor] = None
        if self.pp > 1:
            from rl_b200.parallel.pipeline import PipelineComm

            self._pp_comm = PipelineComm(self.ps)
        self._fp8_scales: dict = {}
        self._sync_weights()  # the rollout copy starts from the initial weights

    def _sync_weights(self) -> None:
        """Refresh the rollout weights; with an fp8 rollout also point the rollout
        model at the quantised weights (scales re-laid-out in place, so captured
        decode graphs keep reading valid buffers)."""
        self.weight_sync.sync()
        ws = self.weight_sync
        if not (self.fp8_rollout and getattr(ws, "fp8", False)):
            return
        from rl_b200.ops.fp8_gemm import mx_weight_scales

        fw = {}
        for name in ws.q_layout:
            q, sc = ws.fp8_weight(name)
            if self.fp8_pow2:
                st = self._fp8_scales.get(name)
                if st is None:
                    st = self._fp8_scales[name] = mx_weight_scales(sc)
                else:
                    st[:, :sc.shape[0]].copy_(sc.t())
                fw[name] = (q, st)
            else:
                fw[name] = (q, sc)
        self.gen_model.fp8_pow2 = self.fp8_pow2
        self.gen_model.fp8_weights = fw

    def _make_weight_sync(self, resharded: bool):
        from rl_b200.weight_sync.colocated import (ColocatedInPlaceSynchronizer, ColocatedReshardSynchronizer,
                                                   LoRAMergeSynchronizer)

        if self.lora is not None:
            if resharded:
                raise NotImplementedError("LoRA with a different rollout TP layout")
            return LoRAMergeSynchronizer(self.lora, self.gen_model)
        if self.pp > 1:
            from rl_b200.weight_sync.colocated import PipelineGatherSynchronizer

            return PipelineGatherSynchronizer(self.model, self.gen_model, self.ps.pp_group, self.ps.pp_ranks,
                                              self.ps.pp_rank)
        if self.nvfp4_rollout:
            from rl_b200.weight_sync.colocated import NVFP4RolloutSynchronizer

            return NVFP4RolloutSynchronizer(self.model, self.gen_model)
        if not resharded and not self.fp8_rollout:
            return ColocatedInPlaceSynchronizer()
        if not resharded:
            # same layout, fp8 rollout weights: quantise this rank's own shard in place
            own = [self.model.flat_param.data_ptr() if r == self.ps.tp_rank else 0 for r in range(self.ps.tp_size)]
            return ColocatedReshardSynchronizer(self.model, self.gen_model, self.ps.tp_group, self.ps.tp_rank,
                                                self.ps.tp_size, peer_ptrs=own if self.device.type == "cuda" else None,
                                                fp8=True, pow2_scales=self.fp8_pow2, copy_bf16=False)
        peer_ptrs = None
        symm = getattr(self.model.flat_param, "_symm", None)
        if symm is not None:
            # symmetric buffers are indexed by global rank; the reshard wants TP-group order
            peer_ptrs = [symm.ptrs[dist.get_global_rank(self.ps.tp_group, r)] for r in range(self.ps.tp_size)]
        return ColocatedReshardSynchronizer(self.model, self.gen_model, self.ps.tp_group, self.ps.tp_rank,
                                            self.ps.tp_size, peer_ptrs=peer_ptrs, fp8=self.fp8_rollout,
                                            pow2_scales=self.fp8_pow2)

    # ------------------------------------------------------------- helpers
    def _plan(self, lengths: list[int], rows: list[int], budget: int) -> list[list[int]]:
        """Sequence-packing plan (list of row lists).  Under expert parallelism the
        ranks of an EP group exchange tokens inside every forward / backward, so
        they must run the SAME number of micro-batches: the plan is padded to the
        group maximum - first by splitting multi-row bins, then with dummy bins
        (negative row ids: the first row again, run with zero loss weight)."""
        bins: list[list[int]] = []
        if rows and getattr(self, "_pair_rows", False):
            # preference data: rows (2i, 2i+1) are a (chosen, rejected) pair and must
            # share a micro-batch, in order; pack pairs as units
            pairs = [(r, r + 1) for r in rows if r % 2 == 0 and r + 1 in set(rows)]
            plen = [lengths[a] + lengths[b] for a, b in pairs]
            budget = max(budget, max(plen))
            packer = get_packer(self.packing_algorithm, bin_capacity=budget,
                                max_sequences_per_bin=self.max_sequences_per_bin)
            for b in packer.pack([max(1, L) for L in plen]):
                bins.append([x for i in sorted(b) for x in pairs[i]])
        elif rows:
            budget = max(budget, max(lengths[r] for r in rows))
            packer = get_packer(self.packing_algorithm, bin_capacity=budget,
                                max_sequences_per_bin=self.max_sequences_per_bin)
            bins = [[rows[i] for i in b] for b in packer.pack([max(1, lengths[r]) for r in rows])]
        if self.microbatch_order == "largest_first":
            bins.sort(key=lambda b: sum(lengths[r] for r in b), reverse=True)
        if self.ps.ep_size > 1 and self.model_cfg.is_moe:
            n = torch.tensor([len(bins)], dtype=torch.int64,
                             device=self.device if self.ps.backend == "nccl" else torch.device("cpu"))
            dist.all_reduce(n, op=dist.ReduceOp.MAX, group=self.ps.ep_group)
            target = int(n.item())
            while len(bins) < target and any(len(b) > 1 for b in bins):
                b = max((b for b in bins if len(b) > 1), key=lambda bb: sum(lengths[r] for r in bb))
                bins.remove(b)
                bins += [b[: len(b) // 2], b[len(b) // 2:]]
            filler = rows[0] if rows else 0
            while len(bins) < target:
                bins.append([-1 - filler])
        return bins

    def _metric_group(self):
        """Group over which per-rank loss partial sums add up: DP, times CP (each
        CP rank scores its own chunks)."""
        if self.ps.cp_size > 1:
            return self.ps.dp_cp_group
        return self.ps.dp_group if self.ps.dp_size > 1 else None

    def _pack_multiple(self) -> int:
        """Packed-token count multiple: the TP size under sequence parallelism, and
        128 x TP when the fused GEMM + reduce-scatter kernel takes the row-parallel
        projections (whole 128-row tiles per rank)."""
        if not self.sequence_parallel:
            return 1
        tp = self.ps.tp_size
        if self.device.type == "cuda" and getattr(self.model, "fused_collectives", False):
            return 128 * tp
        return tp

    def _forward_mb_cp(self, input_ids: torch.Tensor, lengths: list[int], rows: list[int], temperature: float):
        """Context-parallel forward: this rank's two load-balanced chunks of every
        sequence (``rl_b200.parallel.context_parallel``).  Returns local
        (logprob, entropy) and the host scatter map ("cp", seq, pos, lens)."""
        from rl_b200.parallel.context_parallel import cp_layout

        lens = [int(lengths[r]) for r in rows]
        if self.device.type == "cuda":
            # chunks of whole 64-key blocks (overlapped K/V exchange); under SP
            # also 128 x TP tokens per rank for the fused GEMM + collectives
            unit = max(64, 64 * self.ps.tp_size if self.sequence_parallel else 64)
        else:
            unit = max(1, self.ps.tp_size)
        lay = cp_layout(lens, self.ps.cp_size, self.ps.cp_rank, self.device, unit=unit)
        seq = lay.seq_of_local.cpu().numpy()
        pos = lay.positions.cpu().numpy().astype(np.int64)
        L = np.asarray(lens, dtype=np.int64)[seq]
        ids_np = input_ids[rows].numpy() if not input_ids.is_cuda else input_ids[rows].cpu().numpy()
        W = ids_np.shape[1]
        tok = np.where(pos < L, ids_np[seq, np.minimum(pos, W - 1)], 0)
        tgt = np.where(pos + 1 < L, ids_np[seq, np.minimum(pos + 1, W - 1)], 0)
        dev = self.device
        # stays set until the next micro-batch: activation recomputation in the
        # backward pass re-runs the attention with the same layout
        self.model._cp_layout = lay
        hidden = self.model(_to_device(torch.from_numpy(tok), dev), lay.positions, None, lay.max_k)
        h = self.model.lm_input(hidden)
        lp, ent = self._logprobs_from_hidden(h, _to_device(torch.from_numpy(tgt), dev), temperature)
        return lp, ent, ("cp", seq, pos, np.asarray(lens, dtype=np.int64))

    def _forward_mb(self, input_ids: torch.Tensor, lengths: list[int], rows: list[int], temperature: float):
        """Packed forward of ``rows``; returns per-token next-token (logprob, entropy)
        ``[T]`` aligned so that entry j scores token j+1, plus the packing metadata."""
        if self.ps.cp_size > 1:
            return self._forward_mb_cp(input_ids, lengths, rows, temperature)
        flat, pos, cu, max_len, T_real = pack_rows(input_ids, lengths, rows, pad_to_multiple=self._pack_multiple())
        self._set_replay(rows, lengths, flat.numel())
        dev = self.device
        flat_d, pos_d, cu_d = _to_device(flat, dev), _to_device(pos, dev), _to_device(cu, dev)
        targets = torch.empty_like(flat_d)
        targets[:-1] = flat_d[1:]
        targets[-1:] = 0
        hidden = self._run_model(flat_d, pos_d, cu_d, max_len)
        if not self.model.is_last_stage:
            return hidden, None, cu
        h = self.model.lm_input(hidden)
        lp, ent = self._logprobs_from_hidden(h, targets, temperature)
        self._last_cu = cu
        if getattr(self, "_sc_ids", None) is not None:
            self._sc_plk = self._logprobs_at_sampler_topk(h, lp, targets, rows, lengths, temperature)
        return lp, ent, cu

    def _logprobs_at_sampler_topk(self, h, lp, targets, rows, lengths, temperature):
        """Trainer log-probs (with grad) at the rollout sampler's top-k ids of
        every next token, ``[T, k]``: ``logit_v / t - lse`` with the row's
        log-sum-exp recovered from the target's log-prob (no second vocabulary pass)."""
        ids_all = self._sc_ids
        k = ids_all.shape[-1]
        parts = []
        for r in rows:
            L = int(lengths[r])
            nxt = torch.zeros(L, k, dtype=torch.long, device=h.device)
            if L > 1:
                nxt[: L - 1] = ids_all[r, 1:L].to(h.device)
            parts.append(nxt)
        ids = torch.cat(parts)
        T = h.shape[0]
        if ids.shape[0] < T:
            ids = torch.cat([ids, ids.new_zeros(T - ids.shape[0], k)])
        W = self.model.lm_head_weight()
        logit_t = (h * W[targets]).sum(-1).float() / temperature
        lse = logit_t - lp.float()
        return torch.einsum("th,tkh->tk", h, W[ids]).float() / temperature - lse.unsqueeze(-1)

    def _set_replay(self, rows: list, lengths: list, T: int) -> None:
        """Routes of the packed micro-batch for the model's routers (R3), or none."""
        R = self._routes
        if R is None:
            self.model.router_replay = None
            return
        packed = torch.cat([R[r, :lengths[r]] for r in rows])
        if packed.shape[0] < T:
            packed = torch.cat([packed, packed.new_full((T - packed.shape[0],) + tuple(packed.shape[1:]), -1)])
        packed = _to_device(packed, self.device)
        self.model.router_replay = {i: packed[:, i] for i in range(packed.shape[1])}

    def _use_routes(self, data) -> None:
        self._routes = data["routed_experts"] if self.router_replay and "routed_experts" in data else None

    def _end_routes(self) -> None:
        self._routes = None
        self.model.router_replay = None

    def _run_model(self, input_ids, positions, cu_seqlens, max_seqlen):
        """The model (this pipeline stage of it), fed the previous stage's
        activation when there is one."""
        if self.pp > 1:
            return self.model(input_ids, positions, cu_seqlens, max_seqlen, hidden_in=self._pp_in)
        return self.model(input_ids, positions, cu_seqlens, max_seqlen)

    def _pp_shape(self, ids, lengths, rows) -> tuple:
        """Shape of the activation between pipeline stages for a micro-batch."""
        T = pack_rows(ids, lengths, rows, pad_to_multiple=self._pack_multiple())[0].numel()
        if self.sequence_parallel:
            T //= self.ps.tp_size
        return (T, self.model_cfg.hidden_size)

    def _pp_inference(self, plan, ids, lengths, fn) -> None:
        """Forward-only pass of ``plan`` through the pipeline; ``fn(rows, out)``
        consumes the last stage's output of each (non-dummy) micro-batch.  Runs
        the forward steps of the training schedule's plan (same pairing of sends
        and receives)."""
        from rl_b200.parallel.pipeline import _run_plan, plan_1f1b, plan_virtual

        comm = self._pp_comm
        V = self.model.vpp
        mbs = []
        for rows in plan:
            dummy = rows[0] < 0
            mbs.append(([-1 - rows[0]] if dummy else rows, dummy))
        steps = (plan_virtual(comm.n, comm.stage, len(mbs), V, backward=False) if V > 1
                 else plan_1f1b(comm.n, comm.stage, len(mbs), backward=False))

        def forward(i, v, h):
            self.model.chunk = v if V > 1 else None
            self._pp_in = h
            out = fn(*mbs[i])
            self._pp_in = None
            return out

        _run_plan(comm, steps, forward, lambda i: self._pp_shape(ids, lengths, mbs[i][0]), self.dtype,
                  self.device, backward=False)
        self.model.chunk = None

    def _pp_broadcast(self, t: torch.Tensor) -> torch.Tensor:
        """Last stage's tensor to every stage of the pipeline."""
        dev = self.device if self.ps.backend == "nccl" else torch.device("cpu")
        x = t.to(dev).contiguous()
        dist.broadcast(x, src=self.ps.pp_ranks[-1], group=self.ps.pp_group)
        return x.cpu()

    def _pp_share_metrics(self, agg: dict) -> dict:
        obj = [agg]
        dist.broadcast_object_list(obj, src=self.ps.pp_ranks[-1], group=self.ps.pp_group)
        return obj[0]

    def _filtering(self) -> bool:
        gen = self.cfg.get("generation", {}) or {}
        return bool(gen.get("top_k")) or float(gen.get("top_p", 1.0) or 1.0) < 1.0

    def _logprobs_from_hidden(self, h, targets, temperature):
        """Fused LM-head + log-prob (full vocabulary), or - when the rollout samples
        with top-k / top-p - the same filter applied at train time (and, when the
        loss has a KL term, the unfiltered log-probs beside them: the KL compares
        with the unfiltered reference)."""
        grp = self.ps.tp_group if self.ps.tp_size > 1 else None
        gen = self.cfg.get("generation", {}) or {}
        top_k, top_p = gen.get("top_k"), float(gen.get("top_p", 1.0) or 1.0)
        if top_k or top_p < 1.0:
            from rl_b200.ops.fused_linear_logprob import filtered_linear_logprobs

            w = self.model.lm_head_weight()
            if getattr(self, "_need_unfiltered", False):
                self._lp_unfiltered = linear_logprobs(h, w, targets, self.model.vocab_start, temperature, grp,
                                                      self.logprob_chunk)[0]
            return filtered_linear_logprobs(h, w, targets, self.model.vocab_start, temperature, top_k, top_p,
                                            grp, chunk=max(1, min(self.logprob_chunk, 1024)))
        return linear_logprobs(h, self.model.lm_head_weight(), targets, self.model.vocab_start, temperature,
                               grp, self.logprob_chunk)

    def _loss_input(self, loss_fn, ids, lengths, rows, width, temperature):
        """What the loss consumes for one packed micro-batch:
        LOGPROB -> next-token logprobs ``[n, width-1]``;
        VALUE   -> per-token values ``[n, width]`` (value of token i at index i);
        LOGIT   -> full next-token logits ``[n, width-1, V]`` (distillation)."""
        kind = getattr(getattr(loss_fn, "input_type", None), "value", "logprob")
        if kind == "logprob":
            lp, _, cu = self._forward_mb(ids, lengths, rows, temperature)
            if not self.model.is_last_stage:
                return lp  # this stage's output activation
            if isinstance(cu, tuple):
                # the loss sees only this rank's tokens (the others' positions are
                # masked; their ranks contribute them): tokens i+1 scored locally
                one = torch.ones(lp.shape[0], device=lp.device)
                self._cp_owned = self._to_padded(one, cu, len(rows), width)
            return self._to_padded(lp, cu, len(rows), width)
        if self.ps.cp_size > 1:
            raise NotImplementedError("context parallelism supports log-prob losses")
        flat, pos, cu, max_len, _ = pack_rows(ids, lengths, rows, pad_to_multiple=self._pack_multiple())
        self._set_replay(rows, lengths, flat.numel())
        dev = self.device
        hidden = self._run_model(_to_device(flat, dev), _to_device(pos, dev), _to_device(cu, dev), max_len)
        if not self.model.is_last_stage:
            return hidden
        if kind == "value":
            v = self.model.values(hidden)
            return self._to_padded_full(v, cu, len(rows), width)
        logits = self.model.logits(hidden).float() / temperature
        if self.ps.tp_size > 1:
            from rl_b200.parallel.comm import gather_from_sp

            logits = gather_from_sp(logits.t().contiguous(), self.ps.tp_group).t()
        V = logits.shape[-1]
        out = self._to_padded(logits, cu, len(rows), width)  # [n, width-1, V]
        return out.view(len(rows), width - 1, V)

    @staticmethod
    def _to_padded_full(v: torch.Tensor, cu: torch.Tensor, n_rows: int, width: int) -> torch.Tensor:
        """Packed per-token values -> ``[n, width]`` aligned with the input tokens."""
        cu_np = cu.numpy().astype(np.int64)
        lens = np.diff(cu_np)[:n_rows]
        seq = np.repeat(np.arange(n_rows), lens)
        offs = np.arange(int(cu_np[n_rows])) - np.repeat(cu_np[:n_rows], lens)
        N = n_rows * width
        dst = np.full(int(v.shape[0]), N, dtype=np.int64)
        dst[: len(offs)] = seq * width + offs
        di = torch.from_numpy(dst)
        if v.is_cuda:
            di = di.pin_memory().to(v.device, non_blocking=True)
        out = v.new_zeros(N + 1).index_add(0, di, v)
        return out[:N].view(n_rows, width)

    @torch.no_grad()
    def get_values(self, data: BatchedDataDict) -> BatchedDataDict:
        """Value-head outputs ``[B, S]`` (value model / critic)."""
        ids = data["input_ids"]
        B, S = ids.shape
        lengths = self._lengths(data)
        out = torch.zeros(B, S, dtype=torch.float32)
        rows_all = [r for r in range(B) if lengths[r] > 0]
        self._use_routes(data)
        self.model.eval()
        if self.pp > 1:
            def one(rows, dummy):
                width = max(lengths[r] for r in rows)
                v = self._loss_input(_VALUE_INPUT, ids, lengths, rows, width, 1.0)
                if self.model.is_last_stage and not dummy:
                    out[torch.tensor(rows), :width] = v.float().cpu()
                return v

            self._pp_inference(self._plan(lengths, rows_all, self.logprob_mb_tokens), ids, lengths, one)
            self.model.train()
            self._end_routes()
            return BatchedDataDict({"values": self._pp_broadcast(out)})
        for rows in self._plan(lengths, rows_all, self.logprob_mb_tokens):
            if rows[0] < 0:
                continue
            width = max(lengths[r] for r in rows)
            v = self._loss_input(_VALUE_INPUT, ids, lengths, rows, width, 1.0).float().cpu()
            out[torch.tensor(rows), :width] = v
        self.model.train()
        self._end_routes()
        return BatchedDataDict({"values": out})

    @staticmethod
    def _to_padded(lp: torch.Tensor, cu: torch.Tensor, n_rows: int, width: int) -> torch.Tensor:
        """Packed next-token scores -> ``[n, width-1]`` where column i scores token i+1.

        The scatter map is built vectorised on the host from the (host) cu_seqlens
        and copied once; entries that score nothing (each sequence's last token,
        the padding tail) go to a sink slot that is dropped."""
        T = int(lp.shape[0])
        N = n_rows * (width - 1)
        dst = np.full(T, N, dtype=np.int64)
        if isinstance(cu, tuple):  # context parallel: ("cp", seq, pos, lens) of the local tokens
            _, seq, offs, lens = cu
            ok = offs < lens[seq] - 1
            dst[ok] = seq[ok] * (width - 1) + offs[ok]
        else:
            cu_np = cu.numpy().astype(np.int64)
            lens = np.diff(cu_np)[:n_rows]
            seq = np.repeat(np.arange(n_rows), lens)
            offs = np.arange(int(cu_np[n_rows])) - np.repeat(cu_np[:n_rows], lens)
            ok = offs < np.repeat(lens, lens) - 1
            dst[: len(offs)][ok] = seq[ok] * (width - 1) + offs[ok]
        di = torch.from_numpy(dst)
        if lp.is_cuda:
            di = di.pin_memory().to(lp.device, non_blocking=True)
        rest = tuple(lp.shape[1:])
        out = lp.new_zeros((N + 1,) + rest).index_add(0, di, lp)
        return out[:N].view(n_rows, width - 1, *rest)

    def _lengths(self, data: BatchedDataDict) -> list[int]:
        key = "input_lengths" if "input_lengths" in data else "unpadded_sequence_lengths"
        return [int(x) for x in data[key].tolist()]

    # --------------------------------------------------------- logprobs
    @torch.no_grad()
    def get_logprobs(self, data: BatchedDataDict, temperature: Optional[float] = None) -> BatchedDataDict:
        """Logprob of token i at index i (index 0 = 0), ``[B, S]`` fp32 on CPU."""
        temperature = float(temperature if temperature is not None else
                            (self.cfg.get("generation", {}) or {}).get("temperature", 1.0) or 1.0)
        ids = data["input_ids"]
        B, S = ids.shape
        lengths = self._lengths(data)
        out = torch.zeros(B, S, dtype=torch.float32)
        rows_all = [r for r in range(B) if lengths[r] > 0]
        self._use_routes(data)
        self.model.eval()
        if self.pp > 1:
            def one(rows, dummy):
                lp, _, cu = self._forward_mb(ids, lengths, rows, temperature)
                if self.model.is_last_stage and not dummy:
                    out[torch.tensor(rows), 1:] = self._to_padded(lp.float(), cu, len(rows), S).cpu()
                return lp

            self._pp_inference(self._plan(lengths, rows_all, self.logprob_mb_tokens), ids, lengths, one)
            self.model.train()
            self._end_routes()
            return BatchedDataDict({"logprobs": self._pp_broadcast(out)})
        for rows in self._plan(lengths, rows_all, self.logprob_mb_tokens):
            dummy = rows[0] < 0
            rows = [-1 - rows[0]] if dummy else rows
            lp, _, cu = self._forward_mb(ids, lengths, rows, temperature)
            if dummy:
                continue  # padding pass that only keeps the EP group's collectives paired
            padded = self._to_padded(lp.float(), cu, len(rows), S)
            if self.ps.cp_size > 1:  # every CP rank scored its own chunks
                dist.all_reduce(padded, group=self.ps.cp_group)
            out[torch.tensor(rows), 1:] = padded.cpu()
        self.model.train()
        self._end_routes()
        return BatchedDataDict({"logprobs": out})

    @contextlib.contextmanager
    def use_reference_model(self):
        """Swap the reference (initial) weights into the live parameter buffer.
        With LoRA the frozen base IS the reference: the adapters are switched off."""
        if self.lora is not None:
            self.lora.enabled = False
            try:
                yield
            finally:
                self.lora.enabled = True
            return
        if self.ref_flat is None:
            raise RuntimeError("reference model was not initialised")
        flat = self.model.flat_param
        n = self.ref_flat.numel()
        flat[:n].copy_(self.ref_flat)
        self.model.bump_weight_version()
        try:
            yield
        finally:
            # the live bf16 weights are exactly bf16(master): restore by casting
            # the fp32 master shard (no second copy of the model is held)
            self.optimizer.restore_params_from_master()

    @torch.no_grad()
    def get_reference_policy_logprobs(self, data: BatchedDataDict, temperature: Optional[float] = None):
        with self.use_reference_model():
            lp = self.get_logprobs(data, temperature)["logprobs"]
        return BatchedDataDict({"reference_logprobs": lp})

    # ------------------------------------------------------------- train
    def train(self, data: BatchedDataDict, loss_fn, gbs: Optional[int] = None, eval_mode: bool = False,
              temperature: Optional[float] = None, pair_rows: bool = False, prev_from_current: bool = False) -> dict:
        """One or more optimizer steps over ``data`` (this rank's shard).

        ``gbs`` is the LOCAL number of rows per optimizer step (global batch / dp).
        ``pair_rows`` keeps rows (2i, 2i+1) in one micro-batch (preference losses).
        ``prev_from_current``: ``data`` is consumed in ONE optimizer step, so the
        log-probs of the weights before the step are exactly this step's forward
        log-probs; the loss takes them (detached) as ``prev_logprobs`` and the
        separate inference pass is skipped by the caller."""
        if prev_from_current and gbs is not None and gbs < data["input_ids"].shape[0]:
            raise ValueError("prev_from_current needs the whole batch in one optimizer step")
        self._pair_rows = pair_rows
        self._prev_from_current = prev_from_current
        try:
            return self._train(data, loss_fn, gbs, eval_mode, temperature)
        finally:
            self._pair_rows = False
            self._prev_from_current = False

    def _train(self, data: BatchedDataDict, loss_fn, gbs, eval_mode, temperature) -> dict:
        B = data["input_ids"].shape[0]
        gbs = gbs or B
        all_metrics: list[dict] = []
        losses, grad_norms, lrs = [], [], []
        step_extra: dict = {}
        dev_data = None
        for g0 in range(0, B, gbs):
            st = self.begin_train_step(data, loss_fn, rows=range(g0, min(B, g0 + gbs)), eval_mode=eval_mode,
                                       temperature=temperature, _dev_data=dev_data)
            dev_data = st.dev_data
            for i in range(st.num_microbatches):
                self.train_microbatch(st, i)
            res = self.finish_train_step(st, release_grad=False, aggregate=False)
            step_extra = {k: v for k, v in res.items() if k.startswith("moe/")}
            losses.append(res["loss"])
            if not eval_mode:
                grad_norms.append(res["grad_norm"])
                lrs.append(res["lr"])
            all_metrics.extend(st.mb_metrics)
        if self.release_grad_after_train:
            self.optimizer.release_grad_buffer()
        agg = aggregate_metrics(all_metrics, self._metric_group())
        if self.pp > 1:
            agg = self._pp_share_metrics(agg)
        agg.update(step_extra)  # per-step extras of the last step (expert-bias load ratios)
        agg.update({"loss": sum(losses) / max(1, len(losses)), "global_loss": losses,
                    "grad_norm": grad_norms[-1] if grad_norms else 0.0, "lr": lrs[-1] if lrs else 0.0,
                    "moe_aux_loss": self.model.aux_loss()})
        return agg

    # ------------------------------------------- split train API (one step)
    def begin_train_step(self, data: BatchedDataDict, loss_fn, rows=None, eval_mode: bool = False,
                         temperature: Optional[float] = None, _dev_data=None) -> "TrainStepState":
        """Start ONE optimizer step over ``rows`` of ``data`` (default: all rows):
        moves the batch to the device, reduces the global valid-token / sequence
        counts over DP(xCP) and plans the packed micro-batches.  Follow with
        ``train_microbatch(state, i)`` for ``i < state.num_microbatches`` (the
        caller may interleave other work between micro-batches, e.g. an async
        rollout pump) and ``finish_train_step(state)``.

        Reference: the single-controller split train API
        (``begin_train_step`` / ``train_microbatch`` / ``finish_train_step``,
        ``nemo_rl/algorithms/single_controller.py:1-25``)."""
        temperature = float(temperature if temperature is not None else
                            (self.cfg.get("generation", {}) or {}).get("temperature", 1.0) or 1.0)
        ids = data["input_ids"]
        B = ids.shape[0]
        rows = list(rows) if rows is not None else list(range(B))
        lengths = self._lengths(data)
        self.optimizer.ensure_grad_buffer()
        if self.engine.kv_arena is not None and self.engine.arena_dirty:
            self.engine.finish_generation()   # the arena goes back to being gradients
            self.engine.arena_dirty = False
            self.optimizer.zero_grad()
        # the per-token training tensors cross PCIe once (pinned, async) and are
        # sliced on the device; no pageable copy stalls the launch stream later
        dev_data = _dev_data if _dev_data is not None else \
            {k: _to_device(v, self.device) for k, v in data.items()
             if isinstance(v, torch.Tensor) and k != "routed_experts"}  # routes are packed per micro-batch
        g0, n = rows[0], len(rows)
        tok_mask = dev_data["token_mask"][g0:g0 + n, 1:].float()
        smask = dev_data["sample_mask"][g0:g0 + n].float()
        counts = torch.stack([(tok_mask * smask.unsqueeze(-1)).sum(), smask.sum()])
        if self.ps.dp_size > 1:
            # CP ranks hold the same rows: global counts are a sum over data-parallel ranks only
            dist.all_reduce(counts, group=self.ps.dp_group)
        plan = self._plan(lengths, [r for r in rows if lengths[r] > 0], self.train_mb_tokens)
        self.model.aux_loss_scale = 1.0 / max(1, len(plan))
        self._use_routes(data)
        if self._routes is not None and self.pp > 1 and self.model.activation_checkpointing:
            raise NotImplementedError("router replay with pipeline parallelism and activation checkpointing")
        return TrainStepState(ids=ids, lengths=lengths, dev_data=dev_data, loss_fn=loss_fn, plan=plan,
                              gtoks=counts[0], gseqs=counts[1], eval_mode=eval_mode, temperature=temperature,
                              step_loss=torch.zeros((), device=self.device))

    def train_microbatch(self, st: "TrainStepState", i: int) -> dict:
        """Forward + backward of packed micro-batch ``i`` of the step; gradients
        accumulate into the fp32 main-grad buffer.  Returns the (device) metrics.

        Under pipeline parallelism the micro-batches of a step run as one 1F1B
        schedule across the stages: calls for ``i < M - 1`` only count, the last
        call runs the whole schedule (metrics are returned by ``finish_train_step``)."""
        if self.pp > 1:
            st.done += 1
            if i == st.num_microbatches - 1:
                self._pp_train_schedule(st)
            return {}
        arm = (self._overlap_grad_reduce and not st.eval_mode and st.done == st.num_microbatches - 1
               and self.optimizer.begin_overlap())
        if arm:
            self.model.grad_ready_hook = self.optimizer.layer_ready
        try:
            loss, metrics = self._mb_loss(st, i)
            if not st.eval_mode:
                loss.backward()
                self.optimizer._fold_param_grads()
        finally:
            self.model.grad_ready_hook = None
        st.done += 1
        return metrics

    def _pp_train_schedule(self, st: "TrainStepState") -> None:
        from rl_b200.parallel.pipeline import one_f_one_b

        def fwd(i, hidden_in):
            self._pp_in = hidden_in
            try:
                if self.model.is_last_stage:
                    return self._mb_loss(st, i)[0]
                rows = st.plan[i]
                rows = [-1 - rows[0]] if rows[0] < 0 else rows
                width = max(st.lengths[r] for r in rows)
                return self._loss_input(st.loss_fn, st.ids, st.lengths, rows, width, st.temperature)
            finally:
                self._pp_in = None

        def shape(i):
            rows = st.plan[i]
            rows = [-1 - rows[0]] if rows[0] < 0 else rows
            return self._pp_shape(st.ids, st.lengths, rows)

        if self.model.vpp > 1:
            from rl_b200.parallel.pipeline import virtual_pipeline

            def vfwd(i, v, hidden_in):
                self.model.chunk = v
                return fwd(i, hidden_in)

            try:
                virtual_pipeline(self._pp_comm, st.num_microbatches, self.model.vpp, vfwd, shape, self.dtype,
                                 self.device, backward=not st.eval_mode)
            finally:
                self.model.chunk = None
        else:
            one_f_one_b(self._pp_comm, st.num_microbatches, fwd, shape, self.dtype, self.device,
                        backward=not st.eval_mode)
        if not st.eval_mode:
            self.optimizer._fold_param_grads()

    def _mb_loss(self, st: "TrainStepState", i: int):
        """Loss (and metrics) of micro-batch ``i``; accumulates the step loss."""
        mb_rows = st.plan[i]
        dummy = mb_rows[0] < 0
        if dummy:
            mb_rows = [-1 - mb_rows[0]]
        width = max(st.lengths[r] for r in mb_rows)
        self._need_unfiltered = float(getattr(st.loss_fn, "kl_coef", 0.0) or 0.0) != 0.0 and self._filtering() \
            and self.ps.cp_size == 1
        self._lp_unfiltered = None
        self._sc_plk = None
        if getattr(st.loss_fn, "score_centering", False):
            if self.ps.tp_size > 1 or self.ps.cp_size > 1 or self._filtering():
                raise NotImplementedError("score centering needs TP = CP = 1 and no top-k / top-p filtering")
            self._sc_ids = st.dev_data["sampler_topk_token_ids"]
        try:
            curr = self._loss_input(st.loss_fn, st.ids, st.lengths, mb_rows, width, st.temperature)
        finally:
            self._need_unfiltered = False
            self._sc_ids = None
        ridx = torch.tensor(mb_rows, dtype=torch.long).pin_memory().to(self.device, non_blocking=True) \
            if self.device.type == "cuda" else torch.tensor(mb_rows, dtype=torch.long)
        mb = BatchedDataDict({k: (v.index_select(0, ridx)[:, :width] if v.dim() >= 2 else v.index_select(0, ridx))
                              for k, v in st.dev_data.items()})
        if self._lp_unfiltered is not None:
            mb["curr_logprobs_unfiltered"] = self._to_padded(self._lp_unfiltered, self._last_cu, len(mb_rows), width)
            self._lp_unfiltered = None
        if self._sc_plk is not None:
            mb["policy_logprobs_at_sampler_topk"] = self._to_padded(self._sc_plk, self._last_cu, len(mb_rows), width)
            self._sc_plk = None
        if getattr(self, "_prev_from_current", False) and "prev_logprobs" in mb:
            prev = mb["prev_logprobs"].clone()
            prev[:, 1:width] = curr.detach().to(prev.dtype)
            mb["prev_logprobs"] = prev
        if self.ps.cp_size > 1:
            if getattr(st.loss_fn, "loss_type", None) is not None and \
                    getattr(st.loss_fn.loss_type, "value", "") == "sequence_level":
                raise NotImplementedError("sequence-level losses under context parallelism")
            tm = mb["token_mask"].clone()
            tm[:, 1:] = tm[:, 1:] * self._cp_owned.to(tm.dtype)
            mb["token_mask"] = tm
        loss, metrics = st.loss_fn(curr, mb, st.gseqs, st.gtoks)
        if dummy:
            # zero-weight pass: keeps the EP group's all-to-alls paired, adds nothing
            loss = loss * 0.0
            metrics = {}
        st.step_loss += loss.detach()
        st.mb_metrics.append(metrics)
        return loss, metrics

    def finish_train_step(self, st: "TrainStepState", release_grad: Optional[bool] = None,
                          aggregate: bool = True) -> dict:
        """Optimizer step (or gradient reset in eval mode) and the step's metrics."""
        if st.done != st.num_microbatches:
            raise RuntimeError(f"finish_train_step after {st.done}/{st.num_microbatches} micro-batches")
        self._end_routes()
        out: dict = {}
        if not st.eval_mode:
            opt_stats = self.optimizer.step()
            out.update(grad_norm=opt_stats["grad_norm"], lr=opt_stats["lr"])
            if self._expert_bias_rate > 0:
                out.update(self.model.update_expert_bias(
                    self._expert_bias_rate, self.ps.dp_cp_group if self.ps.cp_size > 1 else self.ps.dp_group))
        else:
            self.optimizer.zero_grad()
        red = self._metric_group()
        if red is not None:
            dist.all_reduce(st.step_loss, group=red)
        if self.pp > 1:  # only the last stage computed a loss
            dist.all_reduce(st.step_loss, group=self.ps.pp_group)
        out["loss"] = float(st.step_loss)
        if self.device.type == "cuda":
            # a kernel that gave up a bounded wait (peer flag, pipeline barrier) fails the step here
            from rl_b200.ops._ext import check_device_errors

            check_device_errors()
        if release_grad if release_grad is not None else self.release_grad_after_train:
            self.optimizer.release_grad_buffer()
        if aggregate:
            agg = aggregate_metrics(st.mb_metrics, self._metric_group())
            if self.pp > 1:
                agg = self._pp_share_metrics(agg)
            agg.update(out)
            agg["moe_aux_loss"] = self.model.aux_loss()
            return agg
        return out

    # ------------------------------------------------ quantisation-aware training
    @torch.no_grad()
    def calibrate_quantizers(self, data: BatchedDataDict) -> dict:
        """Record every quantised layer's input amax over forwards of ``data``
        (the calibration pass of fake-quantised training); returns the stats.
        Reference: ``_quantize`` of the ModelOpt quantised policy worker
        (``nemo_rl/modelopt/models/policy/workers/megatron_quant_policy_worker.py:195``)."""
        q = self.model.qat
        if q is None:
            raise RuntimeError("policy.quant_cfg is not set")
        q.calibrating = True
        try:
            self.get_logprobs(data)
        finally:
            q.calibrating = False
        return q.quantizer_stats()

    @torch.no_grad()
    def calibrate_qkv_fp8_scales(self, data: BatchedDataDict, margin: float = 1.0) -> dict:
        """Per-layer fp8 KV-cache scales (``amax * margin / 448`` of the rotated
        keys and the values over forwards of ``data``), installed in the rollout
        engine.  Reference: ``calibrate_qkv_fp8_scales``
        (``nemo_rl/models/policy/interfaces.py:145``)."""
        m = self.gen_model
        m.kv_amax = {}
        try:
            lengths = self._lengths(data)
            rows = [r for r in range(len(lengths)) if lengths[r] > 0]
            for mb in self._plan(lengths, rows, self.logprob_mb_tokens):
                mb = [-1 - mb[0]] if mb[0] < 0 else mb
                flat, pos, cu, max_len, _ = pack_rows(data["input_ids"], lengths, mb, pad_to_multiple=1)
                m(_to_device(flat, self.device), _to_device(pos, self.device), _to_device(cu, self.device), max_len)
            amax = m.kv_amax
        finally:
            m.kv_amax = None
        L = m.cfg.num_layers
        ks = [max(float(amax[i][0]) * margin / 448.0, 1e-8) if i in amax else 1.0 for i in range(L)]
        vs = [max(float(amax[i][1]) * margin / 448.0, 1e-8) if i in amax else 1.0 for i in range(L)]
        if self.ps.tp_size > 1:  # one scale per layer across the TP shards
            t = torch.tensor(ks + vs, dtype=torch.float64, device=self.device if self.ps.backend == "nccl" else "cpu")
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.ps.tp_group)
            ks, vs = t[:L].tolist(), t[L:].tolist()
        self.engine.set_kv_scales(ks, vs)
        return {f"layer_{i}": {"k_scale": ks[i], "v_scale": vs[i]} for i in range(L)}

    def get_quantizer_stats(self) -> dict:
        return self.model.qat.quantizer_stats() if self.model.qat is not None else {}

    # -------------------------------------------------------- generation
    def generate(self, data: BatchedDataDict, greedy: bool = False) -> BatchedDataDict:
        """Roll out ``data``.  With rollout TP 1 under training TP ``t`` the TP peers
        (which hold identical data) each generate every t-th row with their full
        rollout copy and exchange the results, so every peer returns the whole
        batch (identical, as the trainer requires).  An fp8 KV cache is
        calibrated on the first batch it serves."""
        if self.engine.kv_dtype == torch.float8_e4m3fn and self.engine.kv_scales is None:
            self.calibrate_qkv_fp8_scales(data)
        if self.pp > 1:
            # every stage holds the whole rollout model and the same rows: split them
            t, r, grp = self.pp, self.ps.pp_rank, self.ps.pp_group
        elif self.gen_tp == self.ps.tp_size or self.ps.tp_size == 1:
            out = self.engine.generate(data, greedy=greedy)
            if self.device.type == "cuda":
                from rl_b200.ops._ext import check_device_errors

                check_device_errors()
            return out
        else:
            t, r, grp = self.ps.tp_size, self.ps.tp_rank, self.ps.tp_group
        B = data.size
        rows = list(range(r, B, t))
        part = self.engine.generate(data.select_indices(rows), greedy=greedy) if rows else None
        part = BatchedDataDict({k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in part.items()}) \
            if part is not None else None
        parts = [None] * t
        dist.all_gather_object(parts, part, group=grp)
        order = [i for q in range(t) for i in range(q, B, t)]
        out = BatchedDataDict.from_batches([p for p in parts if p is not None], pad_value_dict={"routed_experts": -1})
        out.reorder_data(order)
        return out

    def prepare_for_generation(self, num_seqs: Optional[int] = None) -> bool:
        return self.engine.prepare_for_generation(num_seqs)

    def finish_generation(self) -> bool:
        return self.engine.finish_generation()

    def prepare_for_training(self) -> None:
        self.model.train()

    def prepare_for_lp_inference(self) -> None:
        self.model.eval()

    def train_draft(self, data: BatchedDataDict, max_tokens: int = 8192) -> float:
        """One online step of the speculative draft: next-token cross-entropy on the
        rollout sequences (teacher forcing on what the target generated), the
        draft's equivalent of the reference's online Eagle3 / MTP draft training
        (``nemo_rl/models/policy/draft_config.py:64``).  Returns the loss."""
        if self.draft is None:
            return 0.0
        if self.draft_kind in ("eagle3", "dflash"):
            return self._train_eagle3(data, max_tokens)
        lengths = self._lengths(data)
        rows = [r for r in range(len(lengths)) if lengths[r] > 1]
        tot, sel = 0, []
        for r in rows:
            if tot + lengths[r] > max_tokens and sel:
                break
            sel.append(r)
            tot += lengths[r]
        if not sel:
            return 0.0
        flat, pos, cu, max_len, _ = pack_rows(data["input_ids"], lengths, sel, pad_to_multiple=1)
        dev = self.device
        flat_d = _to_device(flat, dev)
        self.draft.train()
        hidden = self.draft(flat_d, _to_device(pos, dev), _to_device(cu, dev), max_len)
        logits = self.draft.logits(hidden).float()
        if self.draft.ps.tp_size > 1:
            from rl_b200.parallel.comm import gather_from_sp

            logits = gather_from_sp(logits.t().contiguous(), self.draft.ps.tp_group).t()
        tgt = torch.empty_like(flat_d)
        tgt[:-1] = flat_d[1:]
        last = torch.zeros_like(flat_d, dtype=torch.bool)
        last[(_to_device(cu[1:], dev) - 1).long()] = True
        loss = torch.nn.functional.cross_entropy(logits[~last], tgt[~last])
        self._draft_opt.zero_grad(set_to_none=True)
        loss.backward()
        self._draft_opt.step()
        return float(loss.detach())

    def _train_eagle3(self, data: BatchedDataDict, max_tokens: int) -> float:
        """One Eagle3 step: a no-grad policy forward over the rollout sequences
        captures the feature layers, then the head learns the token two positions
        ahead of each feature (``Eagle3Draft.train_loss``); ``loss_weight`` scales
        the loss.  Returns the unweighted loss."""
        lengths = self._lengths(data)
        sel, tot = [], 0
        for r in range(len(lengths)):
            if lengths[r] < 3:
                continue
            if tot + lengths[r] > max_tokens and sel:
                break
            sel.append(r)
            tot += lengths[r]
        if not sel:
            return 0.0
        flat, pos, cu, max_len, _ = pack_rows(data["input_ids"], lengths, sel, pad_to_multiple=1)
        dev = self.device
        flat_d, pos_d, cu_d = _to_device(flat, dev), _to_device(pos, dev), _to_device(cu, dev)
        m = self.gen_model
        with torch.no_grad():
            m.capture_layers, m.captured = self.draft.aux_layers, None
            try:
                was = m.training
                m.eval()
                m(flat_d, pos_d, cu_d, max_len)
                feats = torch.cat([m.captured[i] for i in self.draft.aux_layers], -1)
                m.train(was)
            finally:
                m.capture_layers, m.captured = None, None
            emb = m.embed_full(flat_d)
        # row t: feature t, embedding of token t + 1, label token t + 2 (inside its sequence)
        seq_end = torch.repeat_interleave(cu_d[1:].long(), (cu_d[1:] - cu_d[:-1]).long())
        idx = torch.arange(flat_d.numel(), device=dev)
        mask = idx + 2 < seq_end
        self.draft.train()
        if self.draft_kind == "dflash":
            loss = self.draft.train_loss(torch.roll(emb, -1, 0), feats, flat_d, cu_d,
                                         max_anchors=int(self._draft_anchor_cap), seed=self._draft_steps)
        else:
            loss = self.draft.train_loss(torch.roll(emb, -1, 0), feats, torch.roll(flat_d, -2, 0), mask, pos_d, cu_d,
                                         max_len)
        self._draft_steps += 1
        self._draft_opt.zero_grad(set_to_none=True)
        (loss * self.draft_loss_weight).backward()
        self._draft_opt.step()
        return float(loss.detach())

    def refit(self) -> float:
        """Make the rollout weights current.  Colocated and same layout: the
        optimizer step already wrote the bf16 parameters the engine reads, so the
        refit is a no-op apart from invalidating cached state; with a different
        rollout layout (or fp8 rollout weights) the weight synchronizer reshards
        the training shards from the TP peers into the rollout copy."""
        t0 = time.perf_counter()
        self._sync_weights()
        self.engine.update_weights_from_training()
        self.engine.invalidate_kv_cache()
        return time.perf_counter() - t0

    # ------------------------------------------------------- checkpoints
    def save_checkpoint(self, weights_path: str, optimizer_path: Optional[str] = None,
                        fmt: str = "safetensors", async_save: Optional[bool] = None) -> None:
        """``safetensors``: consolidated HF checkpoint (+ per-rank optimizer shards);
        ``torch_dist``: Megatron-style ``iter_0000000/`` DCP checkpoint under Megatron
        parameter names with the optimizer state embedded (when ``optimizer_path``
        is given), loadable at any parallel layout."""
        from rl_b200.models import checkpoint_io as cio

        if self.lora is not None:
            # adapters only (PEFT layout); the frozen base is the model's own checkpoint
            if self.ps.tp_size > 1:
                raise NotImplementedError("saving LoRA adapters under TP > 1")
            if (dist.get_rank() if dist.is_initialized() else 0) == 0:
                self.lora.save_peft(weights_path)
        elif fmt == "torch_dist":
            if async_save is None:
                ck = ((self.cfg.get("megatron_cfg") or {}).get("checkpoint") or {})
                async_save = bool(ck.get("async_save", False))
            self.finalize_async_save()  # one background save at a time
            self._async_save = cio.save_dist_checkpoint(self.model, self.optimizer, weights_path, optimizer_path,
                                                        async_save=bool(async_save))
            return
        else:
            cio.save_hf_checkpoint(self.model, weights_path)
        if optimizer_path is not None:
            os.makedirs(optimizer_path, exist_ok=True)
            rank = dist.get_rank() if dist.is_initialized() else 0
            torch.save(self.optimizer.state_dict(), os.path.join(optimizer_path, f"__{rank}.pt"))

    def load_checkpoint(self, weights_path: str, optimizer_path: Optional[str] = None) -> None:
        from rl_b200.models import checkpoint_io as cio

        if self.lora is not None:
            self.lora.load_peft(weights_path)
            rank = dist.get_rank() if dist.is_initialized() else 0
            opt_file = os.path.join(optimizer_path, f"__{rank}.pt") if optimizer_path else None
            if opt_file and os.path.exists(opt_file):
                self.optimizer.load_state_dict(torch.load(opt_file, map_location="cpu"))
            else:
                with torch.no_grad():
                    for seg in self.optimizer.segments:
                        seg.master.copy_(self.lora.flat_param[seg.s_lo:seg.s_hi])
            self._sync_weights()
            return

        if os.path.isdir(os.path.join(weights_path, "iter_0000000")):
            cio.load_dist_checkpoint(self.model, self.optimizer, weights_path, optimizer_path)
            self.model.bump_weight_version()
            self._sync_weights()
            return
        cio.load_hf_checkpoint(self.model, weights_path)
        self.model.bump_weight_version()
        rank = dist.get_rank() if dist.is_initialized() else 0
        opt_file = os.path.join(optimizer_path, f"__{rank}.pt") if optimizer_path else None
        if opt_file and os.path.exists(opt_file):
            self.optimizer.load_state_dict(torch.load(opt_file, map_location="cpu"))
        else:
            with torch.no_grad():
                for seg in self.optimizer.segments:
                    seg.master.copy_(self.model.flat_param[seg.s_lo:seg.s_hi])
        self._sync_weights()

    def shutdown(self) -> None:
        """Release the rollout engine's captured graphs (they may hold NCCL
        collectives, which must be gone before the process group is destroyed)
        after any background checkpoint write has finished."""
        self.finalize_async_save()
        self.engine.finish_generation()
        self.engine._drop_graphs()
        self.engine._kv_sig = None
        for attr in ("_fused_rs", "_fused_ag"):
            if getattr(self.model, attr, None) is not None:
                getattr(self.model, attr).close()
                setattr(self.model, attr, None)
        for mdl in {id(self.model): self.model, id(self.gen_model): self.gen_model}.values():
            if getattr(mdl, "_decode_ar", None) is not None:
                mdl._decode_ar.close()
                mdl._decode_ar = None
        if getattr(self.model, "_cp_ex", None) is not None:
            self.model._cp_ex.close()
            self.model._cp_ex = None
        if getattr(self.model, "_ep_ex", None) is not None:
            for x in self.model._ep_ex:
                x.close()
            self.model._ep_ex = None
        self.weight_sync.shutdown()

    def offload_before_refit(self) -> None:
        """Nothing to move: the colocated rollout reads the trained weights in place
        (a reshard refit streams them); kept for the reference's call sequence."""

    def offload_after_refit(self) -> None:
        """See ``offload_before_refit``."""

    def recreate_generation_engine(self) -> None:
        """Replace the rollout engine with a fresh one built from the same
        settings (the counterpart of the reference's ``recreate_worker`` for a
        dead generation shard): the old engine's graphs and KV cache are dropped,
        the new one gets the draft model and fp8-KV scales back, and the rollout
        weights are re-synchronised before it serves."""
        old = self.engine
        try:
            old.finish_generation()
            old._drop_graphs()
        except Exception:  # noqa: BLE001 - the engine being replaced may be broken
            pass
        self.engine = RolloutEngine(self.gen_model, self._gen_cfg, **self._engine_spec)
        for attr in ("kv_scales", "capture_error_mode", "record_routes", "record_sampler_topk"):
            if hasattr(old, attr):
                setattr(self.engine, attr, getattr(old, attr))
        if self.draft is not None:
            self.engine.set_draft(self.draft, getattr(self, "_draft_k", None)
                                  or int((self._gen_cfg.get("speculative") or {})["num_speculative_tokens"]))
        self.engine_incarnation = getattr(self, "engine_incarnation", 0) + 1
        self.refit()

    # ------------------------------------------------ async checkpoint saves
    def finalize_async_save(self) -> None:
        """Wait for the background checkpoint write started by ``save_checkpoint``
        (if any) and raise its error."""
        fut = getattr(self, "_async_save", None)
        self._async_save = None
        if fut is not None:
            fut.result()

    def poll_async_save(self) -> bool:
        """Whether no background checkpoint write is pending."""
        fut = getattr(self, "_async_save", None)
        return fut is None or fut.done()

    # ----------------------------------------------------------- host offload
    def offload_to_cpu(self) -> None:
        """Move the training state off the GPU: parameters (the flat buffer's
        storage is released in place, so every parameter view stays valid), the
        optimizer's master weights and moments, the reference weights, the
        gradient buffer and the rollout KV cache.  ``onload`` brings it back."""
        if getattr(self, "_offloaded", None) is not None or self.device.type != "cuda":
            return
        torch.cuda.synchronize()
        saved = {}
        for key, t in (("flat", self.model.flat_param), ("ref", self.ref_flat)):
            if t is None or not t.is_cuda:
                continue
            host = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=True)
            host.copy_(t.detach())
            saved[key] = (t, host, t.untyped_storage().nbytes())
        self.engine.finish_generation()
        self.optimizer.release_grad_buffer()
        self.optimizer.offload()
        for t, _, _ in saved.values():
            t.untyped_storage().resize_(0)
        self._offloaded = saved
        torch.cuda.empty_cache()

    def onload(self) -> None:
        """Undo ``offload_to_cpu``."""
        saved = getattr(self, "_offloaded", None)
        if saved is None:
            return
        for t, host, nbytes in saved.values():
            t.untyped_storage().resize_(nbytes)
            t.detach().copy_(host)
        self.optimizer.onload(self.device)
        self.optimizer.ensure_grad_buffer()
        self._offloaded = None
        torch.cuda.synchronize()


class _ValueInput:
    from rl_b200.algorithms.loss.interfaces import LossInputType as _LIT

    input_type = _LIT.VALUE


_VALUE_INPUT = _ValueInput()

_MIN_KEYS = ("_min",)
_MAX_KEYS = ("_max",)


def aggregate_metrics(metrics: list[dict], group=None) -> dict:
    """Combine per-micro-batch loss metrics: globally-normalised means add up,
    ``*_min`` / ``*_max`` take min / max; then reduce the same way over DP.

    Values may be device tensors: everything is reduced on the device and read
    back with ONE transfer."""
    per_key: dict[str, list] = {}
    dev = None
    for m in metrics:
        for k, v in m.items():
            if isinstance(v, torch.Tensor):
                dev = dev or v.device
                per_key.setdefault(k, []).append(v.detach().reshape(()).to(torch.float64))
            elif isinstance(v, (int, float)):
                per_key.setdefault(k, []).append(float(v))
    if not per_key:
        return {}
    dev = dev or (torch.device("cuda", torch.cuda.current_device())
                  if (group is not None and torch.cuda.is_available()) else torch.device("cpu"))
    kinds = {"min": [], "max": [], "sum": []}
    for k in sorted(per_key):
        kinds["min" if k.endswith(_MIN_KEYS) else "max" if k.endswith(_MAX_KEYS) else "sum"].append(k)
    out: dict[str, float] = {}
    for kind, op in (("min", dist.ReduceOp.MIN), ("max", dist.ReduceOp.MAX), ("sum", dist.ReduceOp.SUM)):
        ks = kinds[kind]
        if not ks:
            continue
        vals = []
        for k in ks:
            t = torch.stack([x if isinstance(x, torch.Tensor) else torch.tensor(x, dtype=torch.float64, device=dev)
                             for x in per_key[k]]).to(dev)
            vals.append(t.min() if kind == "min" else t.max() if kind == "max" else t.sum())
        t = torch.stack(vals)
        if group is not None and dist.is_initialized():
            dist.all_reduce(t, op=op, group=group)
        for k, v in zip(ks, t.tolist()):
            out[k] = v
    return out
