"""Model / optimizer checkpoint formats.

* **HF safetensors** (``model_save_format: safetensors``; reference: Automodel
  ``save_consolidated`` and the converters ``examples/converters/convert_*_to_hf.py``):
  full (unsharded) tensors under Hugging Face parameter names, written by this
  module's own implementation of the safetensors container (8-byte header
  length, JSON header with dtype / shape / byte offsets, raw little-endian data),
  sharded into ``model-0000i-of-0000n.safetensors`` files with a
  ``model.safetensors.index.json`` and a ``config.json``.  Fused tensors are
  split into their HF components (``qkv_proj`` -> ``q_proj``/``k_proj``/
  ``v_proj``, ``gate_up_proj`` -> ``gate_proj``/``up_proj``, per-expert MoE
  weights); tensor/expert-parallel shards are gathered before writing.
* **Megatron torch_dist** (``model_save_format: torch_dist``; reference:
  Megatron-Core ``iter_0000000/`` with ``metadata.json``, ``common.pt`` and DCP
  ``.metadata`` + ``__*_*.distcp`` shards): implemented in
  ``rl_b200.models.megatron_ckpt`` (Megatron parameter names, layer-stacked
  global tensors, optimizer state embedded; loads at any parallel layout).
"""

from __future__ import annotations

import json
import os
import struct
from typing import Iterable, Optional

import torch
import torch.distributed as dist

__all__ = ["save_safetensors", "load_safetensors", "hf_state_dict", "load_hf_state_dict", "save_hf_checkpoint",
           "load_hf_checkpoint", "save_dist_checkpoint", "load_dist_checkpoint"]

_DT = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16", torch.int64: "I64", torch.int32: "I32",
       torch.uint8: "U8", torch.int8: "I8", torch.float8_e4m3fn: "F8_E4M3", torch.bool: "BOOL"}
_DT_INV = {v: k for k, v in _DT.items()}


# ----------------------------------------------------------------- safetensors
def save_safetensors(tensors: dict[str, torch.Tensor], path: str, metadata: Optional[dict] = None) -> None:
    header: dict = {}
    off = 0
    items = []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": _DT[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        items.append(t)
        off += nbytes
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)  # keep the data section 8-byte aligned
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for t in items:
            f.write(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    os.replace(tmp, path)


def load_safetensors(path: str, names: Optional[Iterable[str]] = None) -> dict[str, torch.Tensor]:
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        base = 8 + n
        want = set(names) if names is not None else None
        out = {}
        for name, meta in header.items():
            if name == "__metadata__" or (want is not None and name not in want):
                continue
            a, b = meta["data_offsets"]
            f.seek(base + a)
            buf = bytearray(f.read(b - a))
            dt = _DT_INV[meta["dtype"]]
            t = torch.frombuffer(buf, dtype=torch.uint8) if b > a else torch.empty(0, dtype=torch.uint8)
            out[name] = t.view(dt).reshape(meta["shape"]).clone()
    return out


# ---------------------------------------------------- HF name mapping (full)
def _gather_full(model, sp, t: torch.Tensor) -> torch.Tensor:
    """Reassemble a TP / EP shard into the full tensor (collective on the group)."""
    ps = model.ps
    if sp.ep_dim is not None and sp.tp_dim is not None and ps.tp_size > 1:
        # split experts: TP slices of the FFN first, then the expert shards
        parts = [torch.empty_like(t) for _ in range(ps.tp_size)]
        dist.all_gather(parts, t.contiguous(), group=ps.tp_group)
        if sp.name.endswith("mlp.experts.gate_up_proj"):
            gs, us = zip(*[p.chunk(2, 1) for p in parts])
            t = torch.cat(list(gs) + list(us), 1)
        else:
            t = torch.cat(parts, sp.tp_dim)
        if ps.ep_size > 1:
            parts = [torch.empty_like(t) for _ in range(ps.ep_size)]
            dist.all_gather(parts, t.contiguous(), group=ps.ep_group)
            t = torch.cat(parts, sp.ep_dim)
        return t
    if sp.tp_dim is not None and ps.tp_size > 1:
        parts = [torch.empty_like(t) for _ in range(ps.tp_size)]
        dist.all_gather(parts, t.contiguous(), group=ps.tp_group)
        if sp.name.endswith(("qkv_proj.weight", "qkv_proj.bias")):
            c = model.cfg
            sizes = [model.nq * c.head_dim, model.nkv * c.head_dim, model.nkv * c.head_dim]
            qs, ks, vs = zip(*[torch.split(p, sizes, 0) for p in parts])
            return torch.cat(list(qs) + list(ks) + list(vs), 0)
        if sp.name.endswith("gate_up_proj.weight"):
            gs, us = zip(*[p.chunk(2, 0) for p in parts])
            return torch.cat(list(gs) + list(us), 0)
        return torch.cat(parts, sp.tp_dim)
    if sp.ep_dim is not None and ps.ep_size > 1:
        parts = [torch.empty_like(t) for _ in range(ps.ep_size)]
        dist.all_gather(parts, t.contiguous(), group=ps.ep_group)
        return torch.cat(parts, sp.ep_dim)
    return t


def hf_state_dict(model, dtype: Optional[torch.dtype] = torch.bfloat16) -> dict[str, torch.Tensor]:
    """Full HF-named tensors of the model (collective over TP / EP groups)."""
    c = model.cfg
    out: dict[str, torch.Tensor] = {}
    for sp, p in model.named_flat_params():
        full = _gather_full(model, sp, p.detach())
        if dtype is not None:
            full = full.to(dtype)
        name = sp.name
        if name.endswith(("self_attn.qkv_proj.weight", "self_attn.qkv_proj.bias")):
            kind = name.rsplit(".", 1)[1]
            pre = name[: -len("qkv_proj." + kind)]
            q, k, v = torch.split(full, [c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim,
                                         c.num_kv_heads * c.head_dim], 0)
            out[f"{pre}q_proj.{kind}"], out[f"{pre}k_proj.{kind}"], out[f"{pre}v_proj.{kind}"] = q, k, v
        elif name.endswith("mlp.gate_up_proj.weight"):
            pre = name[: -len("gate_up_proj.weight")]
            g, u = full.chunk(2, 0)
            out[pre + "gate_proj.weight"], out[pre + "up_proj.weight"] = g, u
        elif name.endswith("mlp.experts.gate_up_proj"):
            pre = name[: -len("gate_up_proj")]
            for e in range(full.shape[0]):
                g, u = full[e].chunk(2, 0)
                out[f"{pre}{e}.gate_proj.weight"], out[f"{pre}{e}.up_proj.weight"] = g, u
        elif name.endswith("mlp.experts.down_proj"):
            pre = name[: -len("down_proj")]
            for e in range(full.shape[0]):
                out[f"{pre}{e}.down_proj.weight"] = full[e]
        else:
            out[name] = full
    return out


def load_hf_state_dict(model, sd: dict[str, torch.Tensor]) -> None:
    """Fill the model from full HF-named tensors (each rank slices its shard)."""
    c = model.cfg
    ps = model.ps
    with torch.no_grad():
        for sp, p in model.named_flat_params():
            name = sp.name
            if name.endswith(("self_attn.qkv_proj.weight", "self_attn.qkv_proj.bias")):
                kind = name.rsplit(".", 1)[1]
                pre = name[: -len("qkv_proj." + kind)]
                full = torch.cat([sd[f"{pre}q_proj.{kind}"], sd[f"{pre}k_proj.{kind}"], sd[f"{pre}v_proj.{kind}"]], 0)
            elif name.endswith("mlp.gate_up_proj.weight"):
                pre = name[: -len("gate_up_proj.weight")]
                full = torch.cat([sd[pre + "gate_proj.weight"], sd[pre + "up_proj.weight"]], 0)
            elif name.endswith("mlp.experts.gate_up_proj"):
                pre = name[: -len("gate_up_proj")]
                full = torch.stack([torch.cat([sd[f"{pre}{e}.gate_proj.weight"], sd[f"{pre}{e}.up_proj.weight"]], 0)
                                    for e in range(c.num_experts)])
            elif name.endswith("mlp.experts.down_proj"):
                pre = name[: -len("down_proj")]
                full = torch.stack([sd[f"{pre}{e}.down_proj.weight"] for e in range(c.num_experts)])
            elif name == "lm_head.weight" and name not in sd:
                full = sd["model.embed_tokens.weight"]
            else:
                full = sd[name]
            p.copy_(model.shard_param(sp, full).to(p.dtype).view(sp.shape))


def save_hf_checkpoint(model, path: str, max_shard_bytes: int = 5 << 30) -> None:
    """Consolidated HF checkpoint (rank 0 writes; all ranks join the gathers).
    Under pipeline parallelism the stages' tensors are gathered to rank 0 over
    the pipeline group of the first TP / CP / DP coordinate."""
    sd = hf_state_dict(model)
    ps = model.ps
    if ps.pp_size > 1 and ps.tp_rank == 0 and ps.cp_rank == 0 and ps.dp_rank == 0:
        parts = [None] * ps.pp_size if ps.pp_rank == 0 else None
        dist.gather_object({k: v.cpu() for k, v in sd.items()}, parts, dst=ps.pp_ranks[0], group=ps.pp_group)
        if ps.pp_rank == 0:
            sd = {}
            for part in parts:
                sd.update(part)
    rank0 = (not dist.is_initialized()) or dist.get_rank() == 0
    if not rank0:
        return
    os.makedirs(path, exist_ok=True)
    shards: list[dict] = [{}]
    size = 0
    for k, v in sd.items():
        nb = v.numel() * v.element_size()
        if size + nb > max_shard_bytes and shards[-1]:
            shards.append({})
            size = 0
        shards[-1][k] = v
        size += nb
    n = len(shards)
    weight_map = {}
    for i, sh in enumerate(shards):
        fname = f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_safetensors(sh, os.path.join(path, fname), {"format": "pt"})
        for k in sh:
            weight_map[k] = fname
    total = sum(v.numel() * v.element_size() for v in sd.values())
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(model.cfg.to_hf_config(), f, indent=1)


def load_hf_checkpoint(model, path: str) -> None:
    idx = os.path.join(path, "model.safetensors.index.json")
    sd: dict[str, torch.Tensor] = {}
    if os.path.exists(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
    else:
        files = [f for f in os.listdir(path) if f.endswith(".safetensors")]
    for fn in files:
        sd.update(load_safetensors(os.path.join(path, fn)))
    load_hf_state_dict(model, sd)


# ------------------------------------------------------- sharded dist format
def save_dist_checkpoint(model, optimizer, weights_dir: str, optim_dir: Optional[str], async_save: bool = False):
    """Megatron ``torch_dist`` checkpoint (``iter_0000000/`` of DCP shards under
    Megatron parameter names, ``rl_b200.models.megatron_ckpt``).  As in Megatron,
    the optimizer state is stored inside the weights checkpoint; ``optim_dir``
    only says whether to include it."""
    from rl_b200.models.megatron_ckpt import save_torch_dist

    return save_torch_dist(model, optimizer, weights_dir, save_optimizer=optim_dir is not None, async_save=async_save)


def load_dist_checkpoint(model, optimizer, weights_dir: str, optim_dir: Optional[str]) -> None:
    """Load a ``torch_dist`` checkpoint written at any parallel layout (each rank
    reads only the pieces its own shards need); optimizer state is restored when
    the checkpoint has it and ``optim_dir`` is given, else the moments start
    fresh with the master weights set from the loaded parameters."""
    from rl_b200.models.megatron_ckpt import load_torch_dist

    load_torch_dist(model, optimizer, weights_dir, load_optimizer=optim_dir is not None)
