"""LoRA adapters for the decoder's linear layers.

Reference: ``policy.*_cfg.lora_cfg`` (``examples/configs/grpo_math_1B.yaml:200-212``:
``enabled``, ``dim``, ``alpha``, ``dropout``, ``dropout_position``,
``target_modules`` / ``exclude_modules`` / ``match_all_linear``, ``lora_A_init``)
and ``docs/guides/lora.md``; PEFT adapter checkpoints (``adapter_model.safetensors``
+ ``adapter_config.json``).

Layout: every adapted weight ``W [out, in]`` (this rank's TP shard) gets
``A [r, in]`` and ``B [out, r]`` with ``y = x W^T + (alpha / r) * (x A^T) B^T``;
``B`` starts at zero so the adapted model starts equal to the base.  Under
tensor parallelism the adapter follows its weight: column-parallel weights
(output rows sharded) keep ``A`` replicated and shard ``B``; row-parallel
weights (input columns sharded) shard ``A`` and keep ``B`` replicated, so the
partial products add up in the same reduction as the base GEMM.

All adapter parameters live in ONE flat fp32-master / bf16 buffer laid out
like the model's own, so the same ``FlatAdamW`` steps them; the base weights
are frozen.  The fused q/k/v and gate/up projections have ONE ``A`` each (a
shared down-projection) - exported to PEFT as identical ``lora_A`` for the
split HF modules and the matching row blocks of ``B``, which is the same model.
"""

from __future__ import annotations

import json
import math
import os
from typing import Optional

import torch
import torch.nn as nn

from rl_b200.models.transformer import ParamSpec
from rl_b200.ops.linear import linear

__all__ = ["LoRAConfig", "LoRAAdapters", "TARGETS"]

# module suffix -> (HF module names it stands for, tp sharding of the base weight)
TARGETS = {
    "self_attn.qkv_proj": (("q_proj", "k_proj", "v_proj"), 0),
    "self_attn.o_proj": (("o_proj",), 1),
    "mlp.gate_up_proj": (("gate_proj", "up_proj"), 0),
    "mlp.down_proj": (("down_proj",), 1),
}


class LoRAConfig:
    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        self.enabled = bool(cfg.get("enabled", False))
        self.dim = int(cfg.get("dim", 8))
        self.alpha = float(cfg.get("alpha", 32))
        self.dropout = float(cfg.get("dropout", 0.0))
        self.dropout_position = cfg.get("dropout_position", "post")
        self.target_modules = list(cfg.get("target_modules") or [])
        self.exclude_modules = list(cfg.get("exclude_modules") or [])
        self.match_all_linear = bool(cfg.get("match_all_linear", True))
        self.lora_A_init = cfg.get("lora_A_init", "xavier")
        self.restore_from = cfg.get("restore_from")

    @property
    def scale(self) -> float:
        return self.alpha / self.dim

    def targets(self, suffix: str) -> bool:
        hf_names, _ = TARGETS[suffix]
        if any(n in self.exclude_modules for n in hf_names) or suffix in self.exclude_modules:
            return False
        if self.match_all_linear or not self.target_modules:
            return True
        return any(n in self.target_modules for n in hf_names) or suffix in self.target_modules


class LoRAAdapters:
    """Adapter parameters of one model (exposes the flat-buffer surface
    ``FlatAdamW`` expects: ``flat_param``, ``flat_numel``, ``specs``,
    ``expert_offset``, ``named_flat_params``)."""

    def __init__(self, model, cfg: LoRAConfig, seed: int = 0):
        self.model = model
        self.cfg = cfg
        self.scale = cfg.scale
        r = cfg.dim
        tp = model.ps.tp_size
        specs, self.layers = [], {}
        for i in range(model.cfg.num_layers):
            for suffix, (_, tp_dim) in TARGETS.items():
                name = f"model.layers.{i}.{suffix}.weight"
                if name not in model._params or not cfg.targets(suffix):
                    continue
                out_f, in_f = model._params[name].shape
                # column-parallel base: A replicated but its gradient is a partial sum
                # over the output shards (reduce over TP); row-parallel base: B
                # replicated and applied after the rank-r all-reduce, so its gradient
                # is already identical on every TP rank (never reduce)
                a = ParamSpec(name[:-len(".weight")] + ".lora_A.weight", (r, in_f), "lora_a",
                              tp_dim=1 if (tp_dim == 1 and tp > 1) else None,
                              grad_reduce="tp_sum" if tp_dim == 0 else None)
                b = ParamSpec(name[:-len(".weight")] + ".lora_B.weight", (out_f, r), "zeros",
                              tp_dim=0 if (tp_dim == 0 and tp > 1) else None,
                              grad_reduce="none" if tp_dim == 1 else None)
                specs += [a, b]
                self.layers[name] = (a.name, b.name)
        off = 0
        for sp in specs:
            sp.numel = int(math.prod(sp.shape))
            sp.offset = off
            off += (sp.numel + 63) // 64 * 64
        self.specs = specs
        self.flat_numel = off
        self.expert_offset = off
        dev, dt = model.flat_param.device, model.flat_param.dtype
        self.flat_param = torch.zeros(max(off, 64), dtype=dt, device=dev)
        gen = torch.Generator(device=dev)
        self._params: dict[str, nn.Parameter] = {}
        for sp in specs:
            view = self.flat_param[sp.offset: sp.offset + sp.numel].view(sp.shape)
            if sp.init == "lora_a":
                # the full (unsharded) A is drawn from one seed so every TP layout agrees
                gen.manual_seed((seed * 1000003 + (hash_str(sp.name) & 0x7FFFFFFF)) & 0x7FFFFFFFFFFF)
                full_in = sp.shape[1] * (tp if sp.tp_dim == 1 else 1)
                if cfg.lora_A_init == "uniform":
                    bound = 1.0 / math.sqrt(full_in)
                    full = (torch.rand(r, full_in, generator=gen, device=dev) * 2 - 1) * bound
                else:  # xavier uniform
                    bound = math.sqrt(6.0 / (full_in + r))
                    full = (torch.rand(r, full_in, generator=gen, device=dev) * 2 - 1) * bound
                if sp.tp_dim == 1:
                    full = full.chunk(tp, 1)[model.ps.tp_rank]
                view.copy_(full.to(dt))
            p = nn.Parameter(view, requires_grad=True)
            self._params[sp.name] = p
        self.enabled = True

    def named_flat_params(self):
        for sp in self.specs:
            yield sp, self._params[sp.name]

    def parameters(self):
        return [self._params[sp.name] for sp in self.specs]

    def delta(self, weight_name: str, x: torch.Tensor) -> Optional[torch.Tensor]:
        """``scale * (x A^T) B^T`` for an adapted weight, else None."""
        if not self.enabled or weight_name not in self.layers:
            return None
        an, bn = self.layers[weight_name]
        h = x
        if self.cfg.dropout > 0 and self.cfg.dropout_position == "pre" and torch.is_grad_enabled():
            h = torch.nn.functional.dropout(h, self.cfg.dropout)
        y = linear(linear(h, self._params[an]), self._params[bn]) * self.scale
        if self.cfg.dropout > 0 and self.cfg.dropout_position == "post" and torch.is_grad_enabled():
            y = torch.nn.functional.dropout(y, self.cfg.dropout)
        return y

    @torch.no_grad()
    def merged_into(self, dst_model) -> None:
        """Write base + scale * B A into ``dst_model`` (same TP layout as the base)."""
        for sp, p in self.model.named_flat_params():
            dst_model._params[sp.name].copy_(p)
        for wname, (an, bn) in self.layers.items():
            a, b = self._params[an].float(), self._params[bn].float()
            w = dst_model._params[wname]
            w.copy_((w.float() + self.scale * (b @ a)).to(w.dtype))

    # --------------------------------------------------------- checkpoints
    def peft_state_dict(self) -> dict[str, torch.Tensor]:
        """PEFT-style adapter tensors with HF module names (TP shards gathered by
        the caller when tp > 1); fused q/k/v and gate/up are split."""
        c = self.model.cfg
        out = {}
        for wname, (an, bn) in self.layers.items():
            a = self._params[an].detach().float().cpu()
            b = self._params[bn].detach().float().cpu()
            layer = wname.split(".")[2]
            suffix = wname.split(f"layers.{layer}.")[1][: -len(".weight")]
            hf, _ = TARGETS[suffix]
            parent = suffix.split(".")[0]
            if suffix == "self_attn.qkv_proj":
                hd = c.head_dim
                rows = [self.model.nq * hd, self.model.nkv * hd, self.model.nkv * hd]
            elif suffix == "mlp.gate_up_proj":
                rows = [b.shape[0] // 2, b.shape[0] // 2]
            else:
                rows = [b.shape[0]]
            for mod, bb in zip(hf, torch.split(b, rows, 0)):
                pre = f"base_model.model.model.layers.{layer}.{parent}.{mod}"
                out[f"{pre}.lora_A.weight"] = a.contiguous()
                out[f"{pre}.lora_B.weight"] = bb.contiguous()
        return out

    def save_peft(self, path: str) -> None:
        from rl_b200.models.checkpoint_io import save_safetensors

        os.makedirs(path, exist_ok=True)
        save_safetensors(self.peft_state_dict(), os.path.join(path, "adapter_model.safetensors"))
        mods = sorted({m for s, (hf, _) in TARGETS.items() for m in hf
                       if any(f".{s}.weight" in w for w in self.layers)})
        with open(os.path.join(path, "adapter_config.json"), "w") as f:
            json.dump({"peft_type": "LORA", "r": self.cfg.dim, "lora_alpha": self.cfg.alpha,
                       "lora_dropout": self.cfg.dropout, "target_modules": mods, "bias": "none",
                       "task_type": "CAUSAL_LM"}, f, indent=1)

    @torch.no_grad()
    def load_peft(self, path: str) -> None:
        """Load adapters written by ``save_peft`` (shared A per fused module)."""
        from rl_b200.models.checkpoint_io import load_safetensors

        sd = load_safetensors(os.path.join(path, "adapter_model.safetensors"))
        for wname, (an, bn) in self.layers.items():
            layer = wname.split(".")[2]
            suffix = wname.split(f"layers.{layer}.")[1][: -len(".weight")]
            hf, _ = TARGETS[suffix]
            parent = suffix.split(".")[0]
            pres = [f"base_model.model.model.layers.{layer}.{parent}.{m}" for m in hf]
            a = sd[f"{pres[0]}.lora_A.weight"]
            for p in pres[1:]:
                if not torch.equal(sd[f"{p}.lora_A.weight"], a):
                    raise ValueError(f"{p}: split modules with different lora_A cannot map onto the fused {suffix}")
            b = torch.cat([sd[f"{p}.lora_B.weight"] for p in pres], 0)
            self._params[an].copy_(a.to(self._params[an].dtype))
            self._params[bn].copy_(b.to(self._params[bn].dtype))


def hash_str(s: str) -> int:
    h = 2166136261
    for ch in s.encode():
        h = ((h ^ ch) * 16777619) & 0xFFFFFFFF
    return h
