"""Decoder-only transformer (Llama / Qwen3 dense and Qwen3-MoE families) used by
both the trainer and the in-house rollout engine.

B200-first layout decisions
---------------------------
* All parameters of the (TP/EP-local) model live in ONE flat buffer; every
  ``nn.Parameter`` is a view into it.  The fp32 gradient buffer (``main_grad``
  views), the optimizer's master weights and Adam moments mirror the same
  flat layout.  One kernel launch then updates the whole model, distributed
  optimizer shards are plain contiguous ranges, and the colocated refit is the
  bf16 write of that same launch.
* Activations are packed (THD): ``[T, H]`` with ``cu_seqlens``; no padding
  tokens are ever computed.
* The training forward and the rollout prefill/decode paths share weights and
  kernels (RMSNorm, RoPE, SwiGLU, attention), which keeps train/rollout
  log-probabilities consistent (``train/gen_kl_error``).
* Tensor parallelism: column-parallel QKV and gate/up, row-parallel O and down
  projections, vocab-parallel embedding and LM head; optional sequence
  parallelism (residual stream sharded over tokens between TP regions).
* MoE: router (fp32) -> top-k (softmax, optional renormalisation) -> token
  permutation by expert -> grouped expert GEMMs -> weighted combine; experts
  are sharded over the expert-parallel group with an all-to-all exchange.

Reference: the model is built by Megatron-Bridge / MCore in the reference
(``nemo_rl/models/megatron/setup.py:2520``, forward ``nemo_rl/models/megatron/train.py:158``);
the per-layer op sequence is the one in section 3.3 of the survey.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.utils.checkpoint as ckpt

from rl_b200.models.config import ModelConfig
from rl_b200.ops.activation import swiglu
from rl_b200.ops.attention import flash_attn_varlen, flash_attn_varlen_fwd, paged_decode_attention, write_kv_cache
from rl_b200.ops.linear import linear
from rl_b200.ops.norm import add_rms_norm, rms_norm
from rl_b200.ops.rope import apply_rope_qkv, build_rope_cache
from rl_b200.parallel.comm import (all_to_all_autograd, copy_to_tp, gather_from_sp, reduce_from_tp,
                                   reduce_scatter_to_sp, scatter_to_sp)
from rl_b200.parallel.state import ParallelState, single_process_state

__all__ = ["TransformerLM", "ParamSpec", "KVCache", "stage_layers"]


def stage_layers(num_layers: int, pp: int, rank: int, first: Optional[int] = None,
                 last: Optional[int] = None) -> range:
    """Contiguous layer range of pipeline stage ``rank``.  ``first`` / ``last``
    fix the layer counts of the first / last stage (Megatron's
    ``num_layers_in_first_pipeline_stage`` / ``..._last_...``: the embedding
    and the LM head make those stages heavier); the other stages split the rest
    evenly, which must divide.  Without them the split is balanced, earlier
    stages taking the remainder."""
    if pp > 1 and (first is not None or last is not None):
        f = int(first) if first is not None else None
        l_ = int(last) if last is not None else None
        inner = pp - (f is not None) - (l_ is not None)
        rest = num_layers - (f or 0) - (l_ or 0)
        if rest < 0 or (inner == 0 and rest != 0) or (inner > 0 and rest % inner):
            raise ValueError(f"{num_layers} layers cannot be split over {pp} stages with {f} in the first and "
                             f"{l_} in the last stage (the other stages must divide the rest evenly)")
        mid = rest // inner if inner else 0
        sizes = [mid] * pp
        if f is not None:
            sizes[0] = f
        if l_ is not None:
            sizes[-1] = l_
        start = sum(sizes[:rank])
        return range(start, start + sizes[rank])
    base, extra = divmod(num_layers, pp)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


@dataclass
class ParamSpec:
    name: str            # HF-style name, e.g. model.layers.0.self_attn.qkv_proj.weight
    shape: tuple
    init: str            # "normal", "ones", "zeros"
    tp_dim: Optional[int] = None   # dim sharded over TP (None = replicated)
    ep_dim: Optional[int] = None   # dim sharded over EP (experts)
    offset: int = 0
    numel: int = 0
    no_weight_decay: bool = False
    # gradient reduction over TP: None = default rule (replicated params are
    # all-reduced under sequence parallelism), "tp_sum" = always, "none" = never
    grad_reduce: Optional[str] = None


class KVCache:
    """Paged KV cache: per layer ``[num_blocks, block_size, nkv_local, hd]`` for K and V."""

    def __init__(self, num_layers: int, num_blocks: int, block_size: int, nkv: int, hd: int, dtype, device,
                 arena: Optional[torch.Tensor] = None):
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.dtype = dtype
        shape = (num_layers, 2, num_blocks, block_size, nkv, hd)
        # every slot is written before it is read (block 0 is a never-read sink), so
        # the cache is not cleared: allocation is free, no 10+ GB memset per step
        n = 1
        for d in shape:
            n *= d
        elt = torch.empty((), dtype=dtype).element_size()
        if arena is not None and arena.numel() * arena.element_size() >= n * elt:
            # borrow the bytes of a caller-owned buffer (the trainer's fp32 gradient
            # arena, idle while the rollout runs)
            self.storage = arena.view(torch.uint8)[: n * elt].view(dtype).view(shape)
        else:
            self.storage = torch.empty(shape, dtype=dtype, device=device)
        # fp8 caches: per-layer per-tensor scales (cache value = k / k_scale)
        self.k_scales = [1.0] * num_layers
        self.v_scales = [1.0] * num_layers

    def layer(self, i: int):
        return self.storage[i, 0], self.storage[i, 1]

    def scales(self, i: int) -> tuple:
        return self.k_scales[i], self.v_scales[i]

    def nbytes(self) -> int:
        return self.storage.numel() * self.storage.element_size()


class _AuxLossScaler(torch.autograd.Function):
    """Attach an auxiliary loss to an activation: forward is the identity, backward
    injects ``scale * d(aux)`` so the aux loss trains without being added to the
    main loss value (MoE load balancing)."""

    @staticmethod
    def forward(ctx, x, aux, scale):
        ctx.save_for_backward(aux)
        ctx.scale = scale
        return x

    @staticmethod
    def backward(ctx, g):
        (aux,) = ctx.saved_tensors
        return g, torch.full_like(aux, ctx.scale), None


class _EmbedFn(torch.autograd.Function):
    """Vocab-(shard-)local embedding lookup whose backward scatters straight into
    the fp32 ``main_grad`` of the table (no dense bf16 table gradient)."""

    @staticmethod
    def forward(ctx, w, ids, vocab_start, sharded):
        ctx.needs_mask = bool(sharded)
        local = ids - vocab_start
        inside = (local >= 0) & (local < w.shape[0])
        lc = local.clamp(0, w.shape[0] - 1)
        ctx.save_for_backward(lc, inside)
        ctx.w = w
        out = w[lc]
        if ctx.needs_mask:
            out = out * inside.unsqueeze(-1).to(w.dtype)
        return out

    @staticmethod
    def backward(ctx, g):
        lc, inside = ctx.saved_tensors
        w = ctx.w
        g = g * inside.unsqueeze(-1).to(g.dtype)
        main = getattr(w, "main_grad", None)
        if main is not None:
            main.index_add_(0, lc, g.float())
            return None, None, None, None
        dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device).index_add_(0, lc, g.float())
        return dw.to(w.dtype), None, None, None


class TransformerLM(nn.Module):
    def __init__(self, cfg: ModelConfig, pstate: Optional[ParallelState] = None, device=None,
                 dtype: torch.dtype = torch.bfloat16, seed: int = 0, sequence_parallel: bool = False,
                 activation_checkpointing: bool = False, init_std: float = 0.02, num_labels: int = 0,
                 flat_alloc: Optional[Callable[[int, torch.dtype], torch.Tensor]] = None, skip_init: bool = False,
                 expert_tensor_parallel: Optional[int] = None):
        """``flat_alloc(numel, dtype)`` supplies the flat parameter buffer (e.g. a
        view of symmetric memory that TP peers can read over NVLink);
        ``skip_init`` leaves the weights unset (a rollout copy filled by refit);
        ``expert_tensor_parallel`` (Megatron's ``expert_tensor_parallel_size``):
        1 keeps every expert whole on each TP rank, the TP size splits each
        expert's FFN over the TP group (column-parallel gate / up, row-parallel
        down); default: split when sequence parallelism is on (required then)."""
        super().__init__()
        self._flat_alloc = flat_alloc
        self._skip_init = skip_init
        self.num_labels = int(num_labels)  # > 0: value / reward model (scalar head instead of LM head)
        self.cfg = cfg
        self.ps = pstate or single_process_state(torch.device(device) if device else None)
        self.device = torch.device(device) if device is not None else self.ps.device
        self.dtype = dtype
        self.sequence_parallel = sequence_parallel and self.ps.tp_size > 1
        self.activation_checkpointing = activation_checkpointing
        tp, ep = self.ps.tp_size, self.ps.ep_size
        if cfg.num_heads % tp or cfg.num_kv_heads % tp:
            raise ValueError(f"heads ({cfg.num_heads}/{cfg.num_kv_heads}) must divide by tp={tp}")
        if cfg.vocab_size % tp:
            raise ValueError(f"vocab {cfg.vocab_size} must divide by tp={tp}")
        self.nq = cfg.num_heads // tp
        self.nkv = cfg.num_kv_heads // tp
        self.hd = cfg.head_dim
        self.vocab_local = cfg.vocab_size // tp
        self.vocab_start = self.ps.tp_rank * self.vocab_local
        self.etp = 1
        if cfg.is_moe:
            if cfg.num_experts % ep:
                raise ValueError(f"experts {cfg.num_experts} must divide by ep={ep}")
            self.experts_local = cfg.num_experts // ep
            self.expert_start = self.ps.ep_rank * self.experts_local
            etp = int(expert_tensor_parallel) if expert_tensor_parallel else (tp if self.sequence_parallel else 1)
            if etp not in (1, tp):
                raise ValueError(f"expert_tensor_parallel_size {etp} must be 1 or the TP size {tp}")
            if self.sequence_parallel and etp != tp:
                # each TP rank would run whole experts on the gathered tokens, and the
                # sequence-parallel reduce-scatter would add their identical outputs
                raise NotImplementedError("MoE under sequence parallelism needs expert_tensor_parallel_size == "
                                          "tensor_model_parallel_size")
            if cfg.moe_ffn_hidden_size % etp:
                raise ValueError(f"expert ffn {cfg.moe_ffn_hidden_size} must divide by etp={etp}")
            self.etp = etp
        else:
            if cfg.ffn_hidden_size % tp:
                raise ValueError(f"ffn {cfg.ffn_hidden_size} must divide by tp={tp}")
            self.ffn_local = cfg.ffn_hidden_size // tp
        # pipeline parallelism: this rank's contiguous range of layers; the first
        # stage owns the embedding, the last the final norm and the LM / value head
        self.pp_size, self.pp_rank = self.ps.pp_size, self.ps.pp_rank
        # virtual pipeline (interleaved layer assignment): the model is cut into
        # pp * vpp chunks and rank r holds chunks r, r + pp, r + 2 pp, ...; the
        # schedule sets ``chunk`` to the one running (None: the rank as a whole)
        self.vpp = int(cfg.extra.get("virtual_pipeline_model_parallel_size") or 1) if self.pp_size > 1 else 1
        self.chunk: Optional[int] = None
        if self.vpp > 1:
            if cfg.extra.get("num_layers_in_first_pipeline_stage") is not None or \
                    cfg.extra.get("num_layers_in_last_pipeline_stage") is not None:
                raise NotImplementedError("uneven first / last stages with a virtual pipeline")
            if cfg.is_moe:
                raise NotImplementedError("virtual pipeline stages for MoE models")
            self.chunk_ranges = [stage_layers(cfg.num_layers, self.pp_size * self.vpp, v * self.pp_size + self.pp_rank)
                                 for v in range(self.vpp)]
            self.layer_range = [i for r in self.chunk_ranges for i in r]
        else:
            self.layer_range = stage_layers(cfg.num_layers, self.pp_size, self.pp_rank,
                                            cfg.extra.get("num_layers_in_first_pipeline_stage"),
                                            cfg.extra.get("num_layers_in_last_pipeline_stage"))
        self._owns_embed = self.pp_rank == 0
        self._owns_head = self.pp_rank == self.pp_size - 1
        if self.pp_size > 1 and cfg.tie_word_embeddings:
            raise NotImplementedError("tied embeddings under pipeline parallelism")
        self.specs = self._make_specs()
        self._allocate(seed, init_std)
        # one row per position the model is configured for (YaRN configs widen it)
        self.rope_cache = build_rope_cache(min(cfg.max_position_embeddings, 1 << 20), cfg.head_dim,
                                           cfg.rope_theta, cfg.rope_scaling, device=self.device)
        self._aux_losses: list[torch.Tensor] = []
        self.aux_loss_scale = 0.0
        # fused compute+collective kernels for TP + SP (GEMM -> reduce-scatter over NVLink)
        self.fused_collectives = True
        self._fused_rs = None
        self._fused_ag = None
        self._ep_ex = None
        self._cp_ex = None
        self._decode_ar = None
        self._cp_layout = None  # rl_b200.parallel.context_parallel.CPLayout of the current micro-batch
        self.lora = None  # rl_b200.models.lora.LoRAAdapters when LoRA training is on
        # router replay (R3): layer -> [T, k] expert ids the router must use;
        # router_record: layer -> [T, k] expert ids chosen (device tensors)
        self.router_replay: Optional[dict] = None
        self.router_record: Optional[dict] = None
        # aux-loss-free load balancing: per-layer expert bias added to the routing
        # scores for the top-k choice only; tokens per expert of the training
        # forwards are accumulated for the bias update (enable_expert_bias)
        self.expert_bias: Optional[dict] = None
        self._expert_load: dict = {}
        # fp8 rollout: name -> (e4m3 weight, block scales) used by the rollout
        # forwards only (forward_prefill / forward_decode); power-of-two scales in
        # the MN-major layout of the hardware-scaled GEMM when fp8_pow2, else
        # [ceil(N/128), K/128] fp32 scales for the promoting GEMM
        self.fp8_weights: Optional[dict] = None
        self.fp8_pow2 = True
        self._in_rollout = False
        # fp8 training (blockwise recipe): {"pow2": bool} when enabled; quantised
        # weights are cached per parameter until weight_version changes
        self.fp8_train: Optional[dict] = None
        self.qat = None  # rl_b200.models.quantization.QAT (fake-quantised training forward)
        self.kv_amax: Optional[dict] = None  # layer -> (k amax, v amax) while calibrating
        self.weight_version = 0
        self._fp8_cache: dict = {}
        # hidden-state capture (Eagle3 draft features): layer -> residual stream after it
        self.capture_layers: Optional[tuple] = None
        # called with a layer index once that layer's backward is complete (set by
        # the policy worker around the backward whose gradient reduction overlaps)
        self.grad_ready_hook = None
        self.captured: Optional[dict] = None

    # ------------------------------------------------------------------ params
    def _make_specs(self) -> list[ParamSpec]:
        c = self.cfg
        H, hd = c.hidden_size, c.head_dim
        s: list[ParamSpec] = []
        if self.is_first_stage or (c.tie_word_embeddings and self.is_last_stage):
            s.append(ParamSpec("model.embed_tokens.weight", (self.vocab_local, H), "normal", tp_dim=0))
        for i in self.layer_range:
            p = f"model.layers.{i}."
            s.append(ParamSpec(p + "input_layernorm.weight", (H,), "ones", no_weight_decay=True))
            s.append(ParamSpec(p + "self_attn.qkv_proj.weight", ((self.nq + 2 * self.nkv) * hd, H), "normal", tp_dim=0))
            if c.attention_bias:
                s.append(ParamSpec(p + "self_attn.qkv_proj.bias", ((self.nq + 2 * self.nkv) * hd,), "zeros", tp_dim=0,
                                   no_weight_decay=True))
            if c.qk_norm:
                s.append(ParamSpec(p + "self_attn.q_norm.weight", (hd,), "ones", no_weight_decay=True))
                s.append(ParamSpec(p + "self_attn.k_norm.weight", (hd,), "ones", no_weight_decay=True))
            s.append(ParamSpec(p + "self_attn.o_proj.weight", (H, self.nq * hd), "normal_out", tp_dim=1))
            s.append(ParamSpec(p + "post_attention_layernorm.weight", (H,), "ones", no_weight_decay=True))
            if c.is_moe:
                F = c.moe_ffn_hidden_size // self.etp
                split = self.etp > 1
                # with split experts the router's gradient is a per-TP-rank partial sum
                # (each rank scores its FFN slice); without SP nothing else adds it up
                s.append(ParamSpec(p + "mlp.gate.weight", (c.num_experts, H), "normal",
                                   grad_reduce="tp_sum" if split and not self.sequence_parallel else None))
                s.append(ParamSpec(p + "mlp.experts.gate_up_proj", (self.experts_local, 2 * F, H), "normal", ep_dim=0,
                                   tp_dim=1 if split else None))
                s.append(ParamSpec(p + "mlp.experts.down_proj", (self.experts_local, H, F), "normal_out", ep_dim=0,
                                   tp_dim=2 if split else None))
            else:
                s.append(ParamSpec(p + "mlp.gate_up_proj.weight", (2 * self.ffn_local, H), "normal", tp_dim=0))
                s.append(ParamSpec(p + "mlp.down_proj.weight", (H, self.ffn_local), "normal_out", tp_dim=1))
        if self.is_last_stage:
            s.append(ParamSpec("model.norm.weight", (H,), "ones", no_weight_decay=True))
            if self.num_labels > 0:
                # value / reward head (HF ``score`` naming of *ForSequenceClassification)
                s.append(ParamSpec("score.weight", (self.num_labels, H), "normal"))
            elif not c.tie_word_embeddings:
                s.append(ParamSpec("lm_head.weight", (self.vocab_local, H), "normal", tp_dim=0))
        # Flat layout: every dense (non-expert) parameter first, then every expert
        # parameter, so that the two gradient-reduction domains (data parallel vs
        # expert data parallel) are two contiguous segments of one buffer.
        s = [sp for sp in s if sp.ep_dim is None] + [sp for sp in s if sp.ep_dim is not None]
        off = 0
        align = 64  # keep every parameter 128-byte aligned (bf16) for vector / TMA access
        self.expert_offset = None
        for sp in s:
            if sp.ep_dim is not None and self.expert_offset is None:
                self.expert_offset = off
            sp.numel = int(math.prod(sp.shape))
            sp.offset = off
            off += (sp.numel + align - 1) // align * align
        self.flat_numel = off
        if self.expert_offset is None:
            self.expert_offset = off
        return s

    def _allocate(self, seed: int, std: float) -> None:
        if self._flat_alloc is not None:
            self.flat_param = self._flat_alloc(self.flat_numel, self.dtype)
        else:
            self.flat_param = torch.empty(self.flat_numel, dtype=self.dtype, device=self.device)
        self.flat_param.zero_()
        if self._skip_init:
            self._params = {}
            for sp in self.specs:
                p = nn.Parameter(self.flat_param[sp.offset: sp.offset + sp.numel].view(sp.shape), requires_grad=False)
                self._params[sp.name] = p
                self.register_parameter(sp.name.replace(".", "__"), p)
            return
        # random init runs on the model's device (an 8B model initialises in seconds on a B200);
        # the CPU and CUDA streams of one seed differ, every TP/EP layout of one device type agrees
        gen = torch.Generator(device=self.device)
        out_std = std / math.sqrt(2 * self.cfg.num_layers)
        self._params: dict[str, nn.Parameter] = {}
        for sp in self.specs:
            view = self.flat_param[sp.offset: sp.offset + sp.numel].view(sp.shape)
            # Seed per (name, shard) so every TP/EP layout of one seed agrees on the
            # full tensor: generate the FULL tensor's shard deterministically.
            gen.manual_seed((seed * 1000003 + (hash_name(sp.name) & 0x7FFFFFFF)) & 0x7FFFFFFFFFFF)
            if sp.init == "ones":
                view.fill_(1.0)
            elif sp.init == "zeros":
                view.zero_()
            else:
                s = std if sp.init == "normal" else out_std
                full = torch.randn(self.full_shape(sp), generator=gen, dtype=torch.float32, device=self.device) * s
                view.copy_(self.shard_param(sp, full).to(self.dtype))
            p = nn.Parameter(view, requires_grad=True)
            self._params[sp.name] = p
            self.register_parameter(sp.name.replace(".", "__"), p)

    def full_shape(self, sp: ParamSpec) -> list:
        """Shape of the whole (unsharded) tensor of ``sp``."""
        shape = list(sp.shape)
        if sp.ep_dim is not None and self.ps.ep_size > 1:
            shape[sp.ep_dim] *= self.ps.ep_size
        if sp.tp_dim is not None and self.ps.tp_size > 1:
            shape[sp.tp_dim] *= self.ps.tp_size
        return shape

    def shard_param(self, sp: ParamSpec, full: torch.Tensor) -> torch.Tensor:
        """This rank's shard of the whole tensor of ``sp`` (expert slice first, then
        the tensor-parallel slice)."""
        if sp.ep_dim is not None and self.ps.ep_size > 1:
            full = full.chunk(self.ps.ep_size, sp.ep_dim)[self.ps.ep_rank]
        if sp.tp_dim is not None and self.ps.tp_size > 1:
            full = self.shard_full_tensor(sp, full, self.ps.tp_rank, self.ps.tp_size)
        return full

    def shard_full_tensor(self, sp: ParamSpec, full: torch.Tensor, idx: int, n: int) -> torch.Tensor:
        """Slice a full (unsharded) tensor into this rank's shard, honouring the
        fused layouts (QKV rows are [q heads | k heads | v heads]; gate/up rows are
        [gate | up]) so that every shard holds matching heads / FFN columns."""
        c = self.cfg
        if sp.name.endswith(("qkv_proj.weight", "qkv_proj.bias")):
            hd = c.head_dim
            q, k, v = torch.split(full, [c.num_heads * hd, c.num_kv_heads * hd, c.num_kv_heads * hd], 0)
            return torch.cat([q.chunk(n, 0)[idx], k.chunk(n, 0)[idx], v.chunk(n, 0)[idx]], 0)
        if sp.name.endswith("gate_up_proj.weight"):
            g, u = full.chunk(2, 0)
            return torch.cat([g.chunk(n, 0)[idx], u.chunk(n, 0)[idx]], 0)
        if sp.name.endswith("mlp.experts.gate_up_proj") and sp.tp_dim is not None:
            g, u = full.chunk(2, 1)  # [E, gate | up, H]: each TP rank takes matching FFN columns of both
            return torch.cat([g.chunk(n, 1)[idx], u.chunk(n, 1)[idx]], 1)
        dim = sp.tp_dim if sp.tp_dim is not None else sp.ep_dim
        return full.chunk(n, dim)[idx]

    def param(self, name: str) -> nn.Parameter:
        return self._params[name]

    def named_flat_params(self):
        for sp in self.specs:
            yield sp, self._params[sp.name]

    # ------------------------------------------------------------ embeddings
    def embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        w = self._params["model.embed_tokens.weight"]
        if self.ps.tp_size == 1:
            return _EmbedFn.apply(w, input_ids, 0, False)
        x = _EmbedFn.apply(w, input_ids, self.vocab_start, True)
        if self.sequence_parallel:
            return reduce_scatter_to_sp(x, self.ps.tp_group)
        return reduce_from_tp(x, self.ps.tp_group)

    def values(self, hidden: torch.Tensor) -> torch.Tensor:
        """Per-token scalar values ``[T]`` (or ``[T, num_labels]``) from the value head."""
        if self.sequence_parallel:
            hidden = gather_from_sp(hidden, self.ps.tp_group)
        v = linear(hidden, self._params["score.weight"]).float()
        return v.squeeze(-1) if self.num_labels == 1 else v

    def lm_head_weight(self) -> torch.Tensor:
        if self.cfg.tie_word_embeddings:
            return self._params["model.embed_tokens.weight"]
        return self._params["lm_head.weight"]

    # -------------------------------------------------------------- attention
    def _qkv(self, i: int, h: torch.Tensor, positions: torch.Tensor, qkv: Optional[torch.Tensor] = None
             ) -> torch.Tensor:
        """QKV projection (unless ``qkv`` is given), optional q/k RMSNorm, RoPE."""
        p = f"model.layers.{i}."
        if qkv is None:
            qkv = self._col_linear(h, p + "self_attn.qkv_proj.weight")
        if self.cfg.attention_bias:
            qkv = qkv + self._params[p + "self_attn.qkv_proj.bias"].to(qkv.dtype)
        if self.cfg.qk_norm:
            T = qkv.shape[0]
            q, k, v = torch.split(qkv, [self.nq * self.hd, self.nkv * self.hd, self.nkv * self.hd], -1)
            q = rms_norm(q.reshape(T * self.nq, self.hd), self._params[p + "self_attn.q_norm.weight"],
                         self.cfg.rms_eps).view(T, -1)
            k = rms_norm(k.reshape(T * self.nkv, self.hd), self._params[p + "self_attn.k_norm.weight"],
                         self.cfg.rms_eps).view(T, -1)
            qkv = torch.cat([q, k, v], -1)
        out = apply_rope_qkv(qkv, positions, self.rope_cache, self.nq, self.nkv, self.hd)
        if self.kv_amax is not None:
            # fp8 KV-cache calibration: amax of the (rotated) keys and the values
            _, k, v = self._split_heads(out)
            ka, va = k.detach().abs().amax().float(), v.detach().abs().amax().float()
            pk, pv = self.kv_amax.get(i, (ka, va))
            self.kv_amax[i] = (torch.maximum(pk, ka), torch.maximum(pv, va))
        return out

    def _split_heads(self, qkv: torch.Tensor):
        T = qkv.shape[0]
        x = qkv.view(T, self.nq + 2 * self.nkv, self.hd)
        return x[:, : self.nq], x[:, self.nq: self.nq + self.nkv], x[:, self.nq + self.nkv:]

    def _fused_ag_ok(self, h: torch.Tensor) -> bool:
        return (self.ps.tp_size > 1 and self.sequence_parallel and self.fused_collectives and h.is_cuda
                and h.dtype == torch.bfloat16 and h.shape[0] % 128 == 0 and self.lora is None
                and self.fp8_train is None)

    def _ag_linear(self, h_shard: torch.Tensor, name: str) -> torch.Tensor:
        """Column-parallel projection of the SP-sharded input with the all-gather
        fused into the GEMM (``rl_b200.parallel.fused.AllGatherGemm``)."""
        from rl_b200.parallel.fused import AllGatherGemm, column_parallel_ag

        op = self._fused_ag
        if op is None or op.ms_max < h_shard.shape[0] or op.K != h_shard.shape[1]:
            if op is not None:
                op.close()
            op = self._fused_ag = AllGatherGemm(self.ps.tp_group, max(h_shard.shape[0] * self.ps.tp_size, 16384),
                                                h_shard.shape[1])
        return column_parallel_ag(h_shard, self._params[name], op)

    def _attn_block(self, i: int, h: torch.Tensor, positions, cu_seqlens, max_seqlen) -> torch.Tensor:
        p = f"model.layers.{i}."
        if self.ps.cp_size > 1 and self._cp_layout is not None:
            return self._attn_block_cp(i, h, positions)
        if self._fused_ag_ok(h):
            qkv = self._qkv(i, None, positions, qkv=self._ag_linear(h, p + "self_attn.qkv_proj.weight"))
        else:
            if self.sequence_parallel:
                h = gather_from_sp(h, self.ps.tp_group)
            else:
                h = copy_to_tp(h, self.ps.tp_group)
            qkv = self._qkv(i, h, positions)
        q, k, v = self._split_heads(qkv)
        o = flash_attn_varlen(q, k, v, cu_seqlens, max_seqlen, causal=True)
        return self._row_parallel_linear(o.reshape(o.shape[0], -1), self._params[p + "self_attn.o_proj.weight"],
                                         p + "self_attn.o_proj.weight")

    def _attn_block_cp(self, i: int, h: torch.Tensor, positions) -> torch.Tensor:
        """Context parallelism: local query chunks attend to their sequence
        prefixes; keys / values are gathered over the CP group
        (``rl_b200.parallel.context_parallel``)."""
        from rl_b200.parallel.context_parallel import cp_attention, gather_kv_cp

        p = f"model.layers.{i}."
        lay = self._cp_layout
        if self.sequence_parallel:
            h = gather_from_sp(h, self.ps.tp_group)
        else:
            h = copy_to_tp(h, self.ps.tp_group)
        qkv = self._qkv(i, h, positions)
        q, k, v = self._split_heads(qkv)
        if (self.fused_collectives and q.is_cuda and q.dtype == torch.bfloat16
                and all(int(c) % 64 == 0 for c in lay.q_len.tolist())):
            from rl_b200.parallel.context_parallel import CPKVExchange, cp_attention_fused

            ex = self._cp_ex
            E = k.shape[1] * k.shape[2]
            if ex is None or ex.max_rows < k.shape[0] or ex.E != E:
                if ex is not None:
                    ex.close()
                ex = self._cp_ex = CPKVExchange(self.ps.cp_group, max(k.shape[0], 8192), E)
            o = cp_attention_fused(q, k.contiguous(), v.contiguous(), lay, ex, 1.0 / math.sqrt(self.hd))
        else:
            kf = gather_kv_cp(k, lay, self.ps.cp_group)
            vf = gather_kv_cp(v, lay, self.ps.cp_group)
            o = cp_attention(q, kf, vf, lay, 1.0 / math.sqrt(self.hd))
        return self._row_parallel_linear(o.reshape(o.shape[0], -1), self._params[p + "self_attn.o_proj.weight"],
                                         p + "self_attn.o_proj.weight")

    def bump_weight_version(self) -> None:
        """The parameters changed (optimizer step, weight swap, load): cached
        quantised copies are stale."""
        self.weight_version += 1

    def _train_linear(self, x: torch.Tensor, w: torch.Tensor, name: Optional[str]) -> torch.Tensor:
        """Training / log-prob projection: block-scaled e4m3 fprop + dgrad when
        fp8 training is on (and the shape allows it), else bf16."""
        if self.qat is not None and not self._in_rollout and self.qat.applies(name):
            return linear(self.qat.input(name, x), self.qat.weight(name, w))
        if self.fp8_train is not None and name is not None and not self._in_rollout:
            from rl_b200.ops.fp8_linear import fp8_supported, fp8_train_linear

            if fp8_supported(w):
                return fp8_train_linear(x, w, self._fp8_cache, name, self.weight_version,
                                        bool(self.fp8_train.get("pow2", True)))
        return linear(x, w)

    def _lin_infer(self, x: torch.Tensor, name: str) -> torch.Tensor:
        """Rollout-time projection: the block-scaled e4m3 weight when the fp8
        rollout holds one for ``name``, else the bf16 weight."""
        fw = self.fp8_weights
        if fw is not None and self._in_rollout and name in fw and x.shape[-1] % 128 == 0:
            from rl_b200.ops.fp8_gemm import fp8_linear, fp8_linear_mx

            q, sc = fw[name]
            return fp8_linear_mx(x, q, sc) if self.fp8_pow2 else fp8_linear(x, q, sc)
        return linear(x, self._params[name])

    def _col_linear(self, h: torch.Tensor, name: str) -> torch.Tensor:
        """Column-parallel projection (+ LoRA delta when adapters are attached)."""
        if self._in_rollout and self.fp8_weights is not None and self.lora is None:
            return self._lin_infer(h, name)
        y = self._train_linear(h, self._params[name], name if self.lora is None else None)
        if self.lora is not None:
            d = self.lora.delta(name, h)
            if d is not None:
                y = y + d
        return y

    def _row_parallel_out(self, out: torch.Tensor) -> torch.Tensor:
        if self.ps.tp_size == 1:
            return out
        if self.sequence_parallel:
            return reduce_scatter_to_sp(out, self.ps.tp_group)
        return reduce_from_tp(out, self.ps.tp_group)

    def _row_parallel_linear(self, x: torch.Tensor, w: torch.Tensor, name: Optional[str] = None) -> torch.Tensor:
        """Row-parallel projection.  With TP + SP on CUDA the GEMM and its
        reduce-scatter run as ONE fused tcgen05 kernel writing peer tiles over
        NVLink (``rl_b200.parallel.fused``); otherwise GEMM then the collective.
        A LoRA adapter's low-rank product is reduced over TP at rank r (tiny)
        and its full output added after the base reduction."""
        tp = self.ps.tp_size
        if self.lora is not None and self.lora.enabled and name in self.lora.layers:
            an, bn = self.lora.layers[name]
            base = self._row_parallel_out(linear(x, w))
            h = linear(x, self.lora._params[an])
            if tp > 1:
                h = reduce_from_tp(h, self.ps.tp_group)
            y = linear(h, self.lora._params[bn]) * self.lora.scale
            if self.sequence_parallel:
                y = scatter_to_sp(y, self.ps.tp_group)
            return base + y
        if (tp > 1 and self.sequence_parallel and self.fused_collectives and x.is_cuda and self.fp8_train is None
                and x.dtype == torch.bfloat16 and x.shape[0] % (128 * tp) == 0 and w.shape[0] % 32 == 0):
            from rl_b200.parallel.fused import GemmReduceScatter, row_parallel_rs

            if self._fused_rs is None or self._fused_rs.max_rows < x.shape[0] or self._fused_rs.N != w.shape[0]:
                if self._fused_rs is not None:
                    self._fused_rs.close()
                self._fused_rs = GemmReduceScatter(self.ps.tp_group, max(x.shape[0], 16384), w.shape[0])
            return row_parallel_rs(x, w, self._fused_rs)
        return self._row_parallel_out(self._train_linear(x, w, name))

    # -------------------------------------------------------------------- MLP
    def _mlp_block(self, i: int, h: torch.Tensor) -> torch.Tensor:
        if self.cfg.is_moe:
            return self._moe_block(i, h)
        p = f"model.layers.{i}."
        if self._fused_ag_ok(h):
            gu = self._ag_linear(h, p + "mlp.gate_up_proj.weight")
        else:
            if self.sequence_parallel:
                h = gather_from_sp(h, self.ps.tp_group)
            else:
                h = copy_to_tp(h, self.ps.tp_group)
            gu = self._col_linear(h, p + "mlp.gate_up_proj.weight")
        a = swiglu(gu)
        return self._row_parallel_linear(a, self._params[p + "mlp.down_proj.weight"], p + "mlp.down_proj.weight")

    def enable_expert_bias(self) -> None:
        """Aux-loss-free load balancing (Megatron's ``moe_router_enable_expert_bias``):
        a zero fp32 bias per MoE layer of this rank's stage."""
        E = self.cfg.num_experts
        dev = self.flat_param.device
        self.expert_bias = {i: torch.zeros(E, dtype=torch.float32, device=dev) for i in self.layer_range}
        self._expert_load = {}

    @torch.no_grad()
    def update_expert_bias(self, rate: float, group=None) -> dict:
        """After an optimizer step: ``bias += rate * sign(mean load - load)`` per
        layer, the tokens per expert summed over ``group`` (the ranks routing
        different tokens); returns the max / min relative load for metrics."""
        import torch.distributed as dist

        if self.expert_bias is None or not self._expert_load:
            return {}
        worst, best = 0.0, float("inf")
        for i, load in self._expert_load.items():
            if group is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
                dist.all_reduce(load, group=group)
            mean = load.mean()
            self.expert_bias[i] += rate * torch.sign(mean - load)
            rel = load / mean.clamp_min(1e-9)
            worst, best = max(worst, float(rel.max())), min(best, float(rel.min()))
        self._expert_load = {}
        return {"moe/max_load_ratio": worst, "moe/min_load_ratio": best}

    def route(self, i: int, h: torch.Tensor):
        """Router: fp32 logits -> softmax -> top-k (+ renormalisation); returns
        (topk_weights [T,k] fp32, topk_ids [T,k] int64, probs [T,E] fp32, perm),
        where ``perm`` is (stable expert-grouped order of the T*k assignments,
        tokens per expert) when the native router kernel produced them, else None."""
        from rl_b200.ops.moe_router import router_topk

        c = self.cfg
        w = self._params[f"model.layers.{i}.mlp.gate.weight"]
        rdtype = torch.float64 if c.moe_router_dtype == "fp64" else torch.float32
        logits = torch.matmul(h.to(rdtype), w.to(rdtype).t())
        perm = None
        if self.router_replay is not None and i in self.router_replay:
            probs = torch.softmax(logits, -1)
            # R3: the experts the rollout chose; tokens without a recorded route
            # (negative ids, e.g. the last sampled token) keep the computed top-k
            rep = self.router_replay[i].to(h.device).long()
            ids = torch.topk(probs, c.moe_top_k, dim=-1)[1]
            ids = torch.where(rep[:, :1] >= 0, rep, ids)
            vals = probs.gather(-1, ids)
        elif self.expert_bias is not None:
            # selection on the biased scores, gating weights from the unbiased ones
            probs = torch.softmax(logits, -1)
            bias = self.expert_bias[i].to(probs.dtype)
            ids = torch.topk(probs.detach() + bias, c.moe_top_k, dim=-1)[1]
            vals = probs.gather(-1, ids)
        elif logits.is_cuda and rdtype == torch.float32:
            # one native pass: softmax, top-k, per-expert counts and the grouped order
            probs, ids, counts, order = router_topk(logits, c.moe_top_k)
            vals = probs.gather(-1, ids)
            perm = (order, counts)
        else:
            probs = torch.softmax(logits, -1)
            vals, ids = torch.topk(probs, c.moe_top_k, dim=-1)
        if self.router_record is not None:
            self.router_record[i] = ids.detach().to(torch.int16 if c.num_experts < 32768 else torch.int32)
        if self.expert_bias is not None and torch.is_grad_enabled():
            load = torch.bincount(ids.detach().reshape(-1), minlength=c.num_experts).float()
            self._expert_load[i] = self._expert_load[i] + load if i in self._expert_load else load
        if c.moe_norm_topk_prob:
            vals = vals / vals.sum(-1, keepdim=True)
        return vals.to(torch.float32), ids, probs.to(torch.float32), perm

    def _moe_block(self, i: int, h: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        p = f"model.layers.{i}."
        split = self.etp > 1  # experts' FFN split over TP: every rank adds a partial output
        if self.sequence_parallel:
            h = gather_from_sp(h, self.ps.tp_group)
        elif split:
            h = copy_to_tp(h, self.ps.tp_group)  # backward: the partial input gradients are summed
        T, H = h.shape
        k, E = c.moe_top_k, c.num_experts
        weights, ids, probs, perm = self.route(i, h)
        if c.moe_aux_loss_coef > 0 and torch.is_grad_enabled():
            # Switch-style load balance: E * sum_e f_e * P_e
            if perm is not None:
                counts = perm[1].float()
            else:
                counts = torch.zeros(E, device=h.device, dtype=torch.float32).index_add_(
                    0, ids.reshape(-1), torch.ones(T * k, device=h.device))
            f = counts / max(1, T * k)
            aux = E * (f.detach() * probs.mean(0)).sum() * c.moe_aux_loss_coef
            # split experts: every TP rank holds the same aux loss, whose gradients the
            # TP reductions add up, so each contributes 1 / tp of it
            scale = (self.aux_loss_scale if self.aux_loss_scale else 1.0) / (self.ps.tp_size if split else 1)
            h = _AuxLossScaler.apply(h, aux, scale)
            self._aux_losses.append(aux.detach())
        wgu = self._params[p + "mlp.experts.gate_up_proj"]
        wdn = self._params[p + "mlp.experts.down_proj"]
        if self.ps.ep_size > 1 and self.fused_collectives and h.is_cuda and h.dtype == torch.bfloat16:
            out = self._moe_ep_fused(h, ids, weights, wgu, wdn, perm)
            if self.sequence_parallel:
                out = reduce_scatter_to_sp(out, self.ps.tp_group)
            elif split:
                out = reduce_from_tp(out, self.ps.tp_group)
            return out
        flat_ids = ids.reshape(-1)
        if perm is not None:
            order, counts = perm
        else:
            order = torch.argsort(flat_ids, stable=True)
            counts = torch.bincount(flat_ids, minlength=E)
        token_of = order // k
        xs = h[token_of]                                             # [T*k, H] permuted by expert
        if self.ps.ep_size > 1:
            ys = self._moe_ep_experts(xs, counts, wgu, wdn)
        else:
            ys = grouped_swiglu_mlp(xs, counts, wgu, wdn)
        # combine: out[t] += w[t, j] * y
        wflat = weights.reshape(-1)[order].to(ys.dtype).unsqueeze(-1)
        out = torch.zeros(T, H, dtype=ys.dtype, device=h.device).index_add_(0, token_of, ys * wflat)
        if self.sequence_parallel:
            out = reduce_scatter_to_sp(out, self.ps.tp_group)
        elif split:
            out = reduce_from_tp(out, self.ps.tp_group)
        return out

    def _moe_ep_fused(self, h, ids, weights, wgu, wdn, perm=None):
        """Expert parallelism with the peer-store dispatch / combine kernels
        (``rl_b200.parallel.ep_fused``): rows land grouped by local expert on
        their owner, outputs return to their assignment slot."""
        from rl_b200.parallel.ep_fused import EPExchange, ep_combine, ep_dispatch, make_plan

        T, H = h.shape
        k = ids.shape[1]
        plan = make_plan(ids, self.ps.ep_size, self.ps.ep_rank, self.experts_local, self.ps.ep_group, perm)
        ex = self._ep_ex
        if ex is None or ex[0].cap < plan.R_max or ex[1].cap < plan.TK_max or ex[0].H != H:
            if ex is not None:
                for x in ex:
                    x.close()
            grow = 1.25  # headroom so that routing drift does not re-allocate every step
            ex = self._ep_ex = (EPExchange(self.ps.ep_group, int(plan.R_max * grow) + 128, H),
                                EPExchange(self.ps.ep_group, int(plan.TK_max * grow) + 128, H))
        xr = ep_dispatch(h.contiguous(), plan, ex[0], ex[1])
        y = grouped_swiglu_mlp(xr, plan.counts_local, wgu, wdn)
        ret = ep_combine(y, plan, ex[0], ex[1])
        return (ret.view(T, k, H) * weights.to(ret.dtype).unsqueeze(-1)).sum(1)

    def _moe_ep_experts(self, xs, counts, wgu, wdn):
        """Expert-parallel path: all-to-all tokens to the ranks owning their experts,
        run the local experts, all-to-all back (NCCL baseline of the fused dispatch)."""
        import torch.distributed as dist

        ep, g = self.ps.ep_size, self.ps.ep_group
        El = self.experts_local
        send_per_rank = counts.view(ep, El).sum(-1)
        all_counts = torch.empty(ep * ep * El, dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(all_counts, counts.contiguous(), group=g)
        all_counts = all_counts.view(ep, ep, El)          # [src_rank, dst_rank, local_expert]
        me = self.ps.ep_rank
        recv = all_counts[:, me, :]                       # [src, El]
        send_splits = send_per_rank.tolist()
        recv_splits = recv.sum(-1).tolist()
        xr = all_to_all_autograd(xs, send_splits, recv_splits, g)
        # received rows are grouped by source, then by local expert: regroup by expert
        src_off = torch.cumsum(torch.cat([recv.new_zeros(1), recv.sum(-1)]), 0)
        idx = []
        for e in range(El):
            for s in range(ep):
                start = int(src_off[s]) + int(recv[s, :e].sum())
                idx.append(torch.arange(start, start + int(recv[s, e]), device=xs.device))
        perm = torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long, device=xs.device)
        y = grouped_swiglu_mlp(xr[perm], recv.sum(0), wgu, wdn)
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel(), device=perm.device)
        return all_to_all_autograd(y[inv], recv_splits, send_splits, g)

    # ------------------------------------------------------------ full model
    def _layer(self, i: int, x: torch.Tensor, resid: Optional[torch.Tensor], positions, cu_seqlens, max_seqlen):
        p = f"model.layers.{i}."
        eps = self.cfg.rms_eps
        if resid is None:
            h = rms_norm(x, self._params[p + "input_layernorm.weight"], eps)
            s = x
        else:
            h, s = add_rms_norm(x, resid, self._params[p + "input_layernorm.weight"], eps)
        a = self._attn_block(i, h, positions, cu_seqlens, max_seqlen)
        h2, s2 = add_rms_norm(s, a, self._params[p + "post_attention_layernorm.weight"], eps)
        m = self._mlp_block(i, h2)
        return s2, m

    @property
    def is_first_stage(self) -> bool:
        """Runs the embedding: the first rank (its first chunk under a virtual pipeline)."""
        return self._owns_embed and (self.chunk is None or self.chunk == 0)

    @property
    def is_last_stage(self) -> bool:
        """Runs the final norm and head: the last rank (its last chunk under a virtual pipeline)."""
        return self._owns_head and (self.chunk is None or self.chunk == self.vpp - 1)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, cu_seqlens: torch.Tensor,
                max_seqlen: int, hidden_in: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Packed forward: ``input_ids [T]`` -> final-norm hidden ``[T(/tp if SP), H]``.
        Under pipeline parallelism a non-first stage starts from ``hidden_in`` (the
        previous stage's output) and a non-last stage returns its residual stream."""
        self._aux_losses = []
        # a non-first pipeline stage (or a draft head fed features) starts from hidden_in
        x = hidden_in if hidden_in is not None else self.embed(input_ids)
        resid = None
        layers = self.chunk_ranges[self.chunk] if (self.vpp > 1 and self.chunk is not None) else self.layer_range
        hook = self.grad_ready_hook
        for i in layers:
            if hook is not None and torch.is_grad_enabled() and x.requires_grad:
                # fires once layer i's backward is complete (its first op produces this gradient last)
                x.register_hook(lambda g, i=i, f=hook: f(i))
            if self.activation_checkpointing and torch.is_grad_enabled():
                if resid is None:
                    x, resid = ckpt.checkpoint(self._layer, i, x, None, positions, cu_seqlens, max_seqlen,
                                               use_reentrant=False)
                else:
                    x, resid = ckpt.checkpoint(self._layer, i, x, resid, positions, cu_seqlens, max_seqlen,
                                               use_reentrant=False)
            else:
                x, resid = self._layer(i, x, resid, positions, cu_seqlens, max_seqlen)
            self._capture(i, x, resid)
        if not self.is_last_stage:
            return x if resid is None else x + resid
        h, _ = add_rms_norm(x, resid, self._params["model.norm.weight"], self.cfg.rms_eps)
        return h

    def lm_input(self, hidden: torch.Tensor) -> torch.Tensor:
        """Hidden states entering the vocab-parallel LM head (gathered from SP,
        gradient all-reduced over TP)."""
        if self.sequence_parallel:
            return gather_from_sp(hidden, self.ps.tp_group)
        return copy_to_tp(hidden, self.ps.tp_group)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Vocab-local logits ``[T, V/tp]`` (hidden gathered from SP if needed)."""
        return linear(self.lm_input(hidden), self.lm_head_weight())

    def aux_loss(self) -> float:
        return float(sum(a.item() for a in self._aux_losses)) if self._aux_losses else 0.0

    # ------------------------------------------------------ rollout (no grad)
    @torch.no_grad()
    def forward_prefill(self, input_ids, positions, cu_seqlens, max_seqlen, kv: KVCache, slot_mapping,
                        last_token_index: torch.Tensor, hidden_in: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Prompt prefill: runs the packed prompts, writes K/V into the paged cache,
        returns the final hidden state of each sequence's last token ``[B, H]``.
        ``hidden_in`` replaces the token embeddings (a draft head fed features)."""
        self._in_rollout = True
        try:
            return self._forward_prefill(input_ids, positions, cu_seqlens, max_seqlen, kv, slot_mapping,
                                         last_token_index, hidden_in)
        finally:
            self._in_rollout = False

    def _capture(self, i: int, x: torch.Tensor, resid: Optional[torch.Tensor]) -> None:
        """Record the residual stream after layer ``i`` when it is a capture layer."""
        if self.capture_layers is not None and i in self.capture_layers:
            if self.captured is None:
                self.captured = {}
            self.captured[i] = (x if resid is None else x + resid).detach()

    def _forward_prefill(self, input_ids, positions, cu_seqlens, max_seqlen, kv, slot_mapping, last_token_index,
                         hidden_in=None):
        x = self.embed_full(input_ids) if hidden_in is None else hidden_in
        resid = None
        eps = self.cfg.rms_eps
        for i in range(self.cfg.num_layers):
            p = f"model.layers.{i}."
            if resid is None:
                h = rms_norm(x, self._params[p + "input_layernorm.weight"], eps)
                s = x
            else:
                h, s = add_rms_norm(x, resid, self._params[p + "input_layernorm.weight"], eps)
            qkv = self._qkv(i, h, positions)
            q, k, v = self._split_heads(qkv)
            kc, vc = kv.layer(i)
            write_kv_cache(k, v, kc, vc, slot_mapping, *kv.scales(i))
            o, _ = flash_attn_varlen_fwd(q, k, v, cu_seqlens, max_seqlen, causal=True)
            a = self._tp_sum(self._lin_infer(o.reshape(o.shape[0], -1), p + "self_attn.o_proj.weight"))
            h2, s2 = add_rms_norm(s, a, self._params[p + "post_attention_layernorm.weight"], eps)
            m = self._mlp_infer(i, h2)
            x, resid = s2, m
            self._capture(i, x, resid)
        h, _ = add_rms_norm(x, resid, self._params["model.norm.weight"], eps)
        return h[last_token_index]

    def _decode_ar_op(self, B: int):
        """Fused TP all-reduce + add + RMSNorm for decode (None when not applicable)."""
        if not (self.ps.tp_size > 1 and self.fused_collectives and self.device.type == "cuda"
                and self.dtype == torch.bfloat16):
            return None
        op = self._decode_ar
        if op is None or op.cap < B:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("decode all-reduce buffers must be created before graph capture")
            if op is not None:
                op.close()
            from rl_b200.parallel.fused import DecodeAllReduceNorm

            op = self._decode_ar = DecodeAllReduceNorm(self.ps.tp_group, max(B, 512), self.cfg.hidden_size)
        return op

    @torch.no_grad()
    def forward_decode(self, tokens, positions, kv: KVCache, block_tables, seq_lens, slot_mapping,
                       max_seq_len: int = 0, hidden_in: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step for ``B`` sequences: ``tokens [B]`` -> hidden ``[B, H]``
        (``hidden_in`` replaces the token embeddings)."""
        self._in_rollout = True
        try:
            return self._forward_decode(tokens, positions, kv, block_tables, seq_lens, slot_mapping, max_seq_len,
                                        hidden_in)
        finally:
            self._in_rollout = False

    def _forward_decode(self, tokens, positions, kv, block_tables, seq_lens, slot_mapping, max_seq_len,
                        hidden_in=None):
        ar = self._decode_ar_op(tokens.shape[0]) if not self.cfg.is_moe else None
        if ar is not None:
            return self._forward_decode_fused_ar(tokens, positions, kv, block_tables, seq_lens, slot_mapping,
                                                 max_seq_len, ar, hidden_in)
        x = self.embed_full(tokens) if hidden_in is None else hidden_in
        resid = None
        eps = self.cfg.rms_eps
        for i in range(self.cfg.num_layers):
            p = f"model.layers.{i}."
            if resid is None:
                h = rms_norm(x, self._params[p + "input_layernorm.weight"], eps)
                s = x
            else:
                h, s = add_rms_norm(x, resid, self._params[p + "input_layernorm.weight"], eps)
            qkv = self._qkv(i, h, positions)
            q, k, v = self._split_heads(qkv)
            kc, vc = kv.layer(i)
            ks, vs = kv.scales(i)
            write_kv_cache(k, v, kc, vc, slot_mapping, ks, vs)
            o = paged_decode_attention(q, kc, vc, block_tables, seq_lens, max_seq_len=max_seq_len,
                                       k_scale=ks, v_scale=vs)
            a = self._tp_sum(self._lin_infer(o.reshape(o.shape[0], -1), p + "self_attn.o_proj.weight"))
            h2, s2 = add_rms_norm(s, a, self._params[p + "post_attention_layernorm.weight"], eps)
            m = self._mlp_infer(i, h2)
            x, resid = s2, m
            self._capture(i, x, resid)
        h, _ = add_rms_norm(x, resid, self._params["model.norm.weight"], eps)
        return h

    def _forward_decode_fused_ar(self, tokens, positions, kv, block_tables, seq_lens, slot_mapping, max_seq_len, ar,
                                 hidden_in=None):
        """Decode step with every row-parallel output reduced by the fused
        peer-memory all-reduce + residual add + RMSNorm (no NCCL in the step)."""
        eps = self.cfg.rms_eps
        s = (self.embed_full(tokens) if hidden_in is None else hidden_in).contiguous()  # residual, updated in place
        h = rms_norm(s, self._params["model.layers.0.input_layernorm.weight"], eps)
        L = self.cfg.num_layers
        for i in range(L):
            p = f"model.layers.{i}."
            qkv = self._qkv(i, h, positions)
            q, k, v = self._split_heads(qkv)
            kc, vc = kv.layer(i)
            ks, vs = kv.scales(i)
            write_kv_cache(k, v, kc, vc, slot_mapping, ks, vs)
            o = paged_decode_attention(q, kc, vc, block_tables, seq_lens, max_seq_len=max_seq_len,
                                       k_scale=ks, v_scale=vs)
            a = self._lin_infer(o.reshape(o.shape[0], -1), p + "self_attn.o_proj.weight")
            h2 = ar(a, s, self._params[p + "post_attention_layernorm.weight"], eps)
            gu = self._lin_infer(h2, p + "mlp.gate_up_proj.weight")
            m = self._lin_infer(swiglu(gu), p + "mlp.down_proj.weight")
            w_next = self._params[f"model.layers.{i + 1}.input_layernorm.weight"] if i + 1 < L \
                else self._params["model.norm.weight"]
            h = ar(m, s, w_next, eps)
            self._capture(i, s, None)
        return h

    def embed_full(self, ids: torch.Tensor) -> torch.Tensor:
        """Embedding with a TP all-reduce but never sequence-sharded (rollout path)."""
        w = self._params["model.embed_tokens.weight"]
        if self.ps.tp_size == 1:
            return w[ids]
        local = ids - self.vocab_start
        inside = (local >= 0) & (local < self.vocab_local)
        x = w[local.clamp(0, self.vocab_local - 1)] * inside.unsqueeze(-1).to(w.dtype)
        return self._tp_sum(x)

    def _tp_sum(self, x: torch.Tensor) -> torch.Tensor:
        if self.ps.tp_size > 1:
            import torch.distributed as dist

            dist.all_reduce(x, group=self.ps.tp_group)
        return x

    def _mlp_infer(self, i: int, h: torch.Tensor) -> torch.Tensor:
        p = f"model.layers.{i}."
        if self.cfg.is_moe:
            sp = self.sequence_parallel
            self.sequence_parallel = False
            try:
                return self._moe_block(i, h)
            finally:
                self.sequence_parallel = sp
        gu = self._lin_infer(h, p + "mlp.gate_up_proj.weight")
        return self._tp_sum(self._lin_infer(swiglu(gu), p + "mlp.down_proj.weight"))

    def logits_infer(self, hidden: torch.Tensor) -> torch.Tensor:
        """Full-vocab logits for sampling ``[B, V]`` (TP shards all-gathered)."""
        local = linear(hidden, self.lm_head_weight())
        if self.ps.tp_size == 1:
            return local
        import torch.distributed as dist

        parts = [torch.empty_like(local) for _ in range(self.ps.tp_size)]
        dist.all_gather(parts, local.contiguous(), group=self.ps.tp_group)
        return torch.cat(parts, -1)


def hash_name(name: str) -> int:
    """Stable (process-independent) string hash for per-parameter init seeds."""
    h = 1469598103934665603
    for ch in name.encode():
        h ^= ch
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def grouped_swiglu_mlp(xs: torch.Tensor, counts: torch.Tensor, wgu: torch.Tensor, wdn: torch.Tensor) -> torch.Tensor:
    """Expert FFNs over rows grouped by expert: ``xs [N, H]`` (rows of expert e are
    contiguous, ``counts[e]`` of them), ``wgu [E, 2F, H]``, ``wdn [E, H, F]``."""
    from rl_b200.ops.grouped_gemm import grouped_mm_nt

    gu = grouped_mm_nt(xs, wgu, counts)
    a = swiglu(gu)
    return grouped_mm_nt(a, wdn, counts)
