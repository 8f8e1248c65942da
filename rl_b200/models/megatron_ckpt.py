"""Megatron ``torch_dist`` checkpoints (``iter_0000000/``) written and read with
PyTorch Distributed Checkpoint (DCP).

Layout written (what Megatron-Core's ``dist_checkpointing`` produces with the
``torch_dist`` backend, and what the reference's resume logic probes,
``nemo_rl/utils/checkpoint.py:345-364``)::

    <weights_dir>/latest_checkpointed_iteration.txt      "0"
    <weights_dir>/iter_0000000/metadata.json             {"sharded_backend": "torch_dist", ...}
    <weights_dir>/iter_0000000/common.pt                 non-sharded state (iteration, optimizer
                                                          param groups / step, layout record)
    <weights_dir>/iter_0000000/.metadata                 DCP metadata (global shapes, chunks)
    <weights_dir>/iter_0000000/__<rank>_0.distcp         DCP data files

Tensors carry Megatron-Core parameter names in its layer-stacked form: every
per-layer parameter is ONE global tensor with a leading layer dimension (key
``decoder.layers.self_attention.linear_qkv.weight``, shape ``[L, ...]``), expert
weights add an expert dimension, and the fused QKV rows use Megatron's grouped
order (per KV group: its query heads, then its key head, then its value head);
the gate / up halves of ``linear_fc1`` are ``[all gate rows; all up rows]``.
Optimizer state is saved under ``optimizer.state.{fp32_param,exp_avg,exp_avg_sq}.
<param key>`` with the parameters' global shapes.

How: each rank describes the slice of every global tensor it holds as a list of
rectangular pieces, each backed by a CONTIGUOUS range of its flat buffers (the
bf16 parameter buffer, or an optimizer shard of the fp32 master / moments).  A
tensor-parallel shard is a block of rows or columns; the QKV reordering is a
permutation of head-sized row blocks; a ZeRO optimizer shard cuts parameters at
arbitrary element offsets, which become (partial row, whole rows, partial row)
pieces.  Saving hands those pieces to DCP as write items (replicas are
de-duplicated by DCP's planner); loading asks DCP for exactly the pieces the
LOADING layout needs, so a checkpoint written at one TP / EP / PP / DP layout
loads into any other one, reading only the byte ranges each rank needs and
streaming tensor by tensor (no rank assembles another rank's shard).

Megatron-Core itself is not installed in this image, so the key names, the
stacking and the QKV order follow its documented ``sharded_state_dict`` layout
but have not been loaded by Megatron here; the files are standard DCP and load
with ``torch.distributed.checkpoint`` (see ``read_global_tensor``).
"""

from __future__ import annotations

import json
import os
import re
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
import torch.distributed.checkpoint as dcp
from torch.distributed.checkpoint.default_planner import DefaultLoadPlanner, DefaultSavePlanner
from torch.distributed.checkpoint.metadata import ChunkStorageMetadata, MetadataIndex, TensorProperties
from torch.distributed.checkpoint.planner import LoadPlan, SavePlan, TensorWriteData, WriteItem, WriteItemType
from torch.distributed.checkpoint.planner_helpers import create_read_items_for_chunk_list

__all__ = ["megatron_key", "save_torch_dist", "load_torch_dist", "read_global_tensor", "is_torch_dist_checkpoint",
           "ITER_DIR"]

ITER_DIR = "iter_0000000"
_METADATA = {"sharded_backend": "torch_dist", "sharded_backend_version": 1, "common_backend": "torch",
             "common_backend_version": 1}

_LAYER_RE = re.compile(r"^model\.layers\.(\d+)\.(.+)$")
# per-layer parameter -> key under decoder.layers. (dense / MoE post-attention norm differ)
_LAYER_KEYS = {
    "input_layernorm.weight": "self_attention.linear_qkv.layer_norm_weight",
    "self_attn.qkv_proj.weight": "self_attention.linear_qkv.weight",
    "self_attn.qkv_proj.bias": "self_attention.linear_qkv.bias",
    "self_attn.q_norm.weight": "self_attention.q_layernorm.weight",
    "self_attn.k_norm.weight": "self_attention.k_layernorm.weight",
    "self_attn.o_proj.weight": "self_attention.linear_proj.weight",
    "mlp.gate_up_proj.weight": "mlp.linear_fc1.weight",
    "mlp.down_proj.weight": "mlp.linear_fc2.weight",
    "mlp.gate.weight": "mlp.router.weight",
    "mlp.experts.gate_up_proj": "mlp.experts.experts.linear_fc1.weight",
    "mlp.experts.down_proj": "mlp.experts.experts.linear_fc2.weight",
}
_TOP_KEYS = {"model.embed_tokens.weight": "embedding.word_embeddings.weight",
             "model.norm.weight": "decoder.final_layernorm.weight",
             "lm_head.weight": "output_layer.weight",
             "value_head.weight": "output_layer.weight"}


def megatron_key(name: str, moe: bool) -> tuple[str, Optional[int]]:
    """(Megatron key, layer index or None) of an internal parameter name."""
    m = _LAYER_RE.match(name)
    if m:
        layer, rest = int(m.group(1)), m.group(2)
        if rest == "post_attention_layernorm.weight":
            key = "pre_mlp_layernorm.weight" if moe else "mlp.linear_fc1.layer_norm_weight"
        elif rest in _LAYER_KEYS:
            key = _LAYER_KEYS[rest]
        else:
            key = rest
        return "decoder.layers." + key, layer
    return _TOP_KEYS.get(name, name), None


@dataclass
class _Piece:
    key: str
    global_shape: tuple
    offsets: tuple
    sizes: tuple
    lo: int   # start within the parameter's local flat range
    n: int    # element count (contiguous in the local flat range)


class _ParamMap:
    """Where the rows of one rank's local parameter shard live in the global
    (Megatron-layout) tensor."""

    def __init__(self, model, sp):
        c, ps = model.cfg, model.ps
        moe = bool(getattr(c, "num_experts", 0))
        self.key, layer = megatron_key(sp.name, moe)
        shape = tuple(sp.shape)
        self.one_d = len(shape) == 1
        self.C = shape[-1]
        self.R = 1 if self.one_d else int(torch.Size(shape[:-1]).numel())
        tp, t = ps.tp_size, ps.tp_rank
        lead: tuple = ()
        lead_shape: tuple = ()
        if layer is not None:
            lead, lead_shape = (layer,), (c.num_layers,)
        self.col0 = 0
        name = sp.name
        runs: list[tuple[int, int, tuple, int]] = []  # (local row, rows, leading offsets, global row)
        if sp.ep_dim is not None:
            # experts [E_local, R_e, C]: leading expert index offset by this rank's first expert;
            # split experts (tp_dim set) hold FFN slices: gate / up row blocks or a column block
            e_local, r_e = shape[0], shape[1]
            e0 = ps.ep_rank * e_local if ps.ep_size > 1 else 0
            split = sp.tp_dim is not None and tp > 1
            if split and sp.tp_dim == 1:  # gate_up [E, gate | up, H]
                f_l = r_e // 2
                body = (c.num_experts, 2 * f_l * tp, self.C)
                for e in range(e_local):
                    runs.append((e * r_e, f_l, lead + (e0 + e,), t * f_l))
                    runs.append((e * r_e + f_l, f_l, lead + (e0 + e,), f_l * tp + t * f_l))
            else:
                if split:  # down [E, H, F]: this rank's FFN columns
                    self.col0 = t * self.C
                body = (c.num_experts, r_e, self.C * (tp if split else 1))
                for e in range(e_local):
                    runs.append((e * r_e, r_e, lead + (e0 + e,), 0))
            gshape = lead_shape + body
        elif name.endswith(("qkv_proj.weight", "qkv_proj.bias")):
            hd = c.head_dim
            nq_l, nkv_l = model.nq, model.nkv
            qpg = c.num_heads // c.num_kv_heads
            grp_rows = (qpg + 2) * hd
            for i in range(nq_l):
                gh = t * nq_l + i if tp > 1 else i
                runs.append((i * hd, hd, lead, (gh // qpg) * grp_rows + (gh % qpg) * hd))
            for i in range(nkv_l):
                g = t * nkv_l + i if tp > 1 else i
                runs.append(((nq_l + i) * hd, hd, lead, g * grp_rows + qpg * hd))
                runs.append(((nq_l + nkv_l + i) * hd, hd, lead, g * grp_rows + (qpg + 1) * hd))
            rows_g = c.num_kv_heads * grp_rows
            gshape = lead_shape + ((rows_g,) if self.one_d else (rows_g, self.C))
            if self.one_d:  # bias: rows are elements
                self.one_d, self.R, self.C = False, shape[0], 1
                self._bias = True
        elif name.endswith("gate_up_proj.weight"):
            f_l = shape[0] // 2
            f = f_l * (tp if tp > 1 else 1)
            runs.append((0, f_l, lead, t * f_l if tp > 1 else 0))
            runs.append((f_l, f_l, lead, f + (t * f_l if tp > 1 else 0)))
            gshape = lead_shape + (2 * f, self.C)
        elif sp.tp_dim == 0 and tp > 1:
            runs.append((0, self.R, lead, t * self.R))
            gshape = lead_shape + ((self.R * tp,) + shape[1:])
        elif sp.tp_dim is not None and tp > 1:  # column shard (last dim)
            self.col0 = t * self.C
            runs.append((0, self.R, lead, 0))
            gshape = lead_shape + (shape[:-1] + (self.C * tp,))
        else:
            runs.append((0, self.R, lead, 0))
            gshape = lead_shape + shape
        self.runs = runs
        self.global_shape = tuple(int(x) for x in gshape)
        self.bias_like = getattr(self, "_bias", False)

    def _rect(self, lead: tuple, grow: int, nrows: int, c0: int, ncols: int) -> tuple[tuple, tuple]:
        """Offsets / sizes of a block of rows (and columns) in the global tensor."""
        nd = len(self.global_shape) - len(lead)
        if self.one_d:  # [*lead, C]
            return lead + (self.col0 + c0,), (1,) * len(lead) + (ncols,)
        if self.bias_like:  # [*lead, rows]
            return lead + (grow,), (1,) * len(lead) + (nrows,)
        if nd == 2:
            return lead + (grow, self.col0 + c0), (1,) * len(lead) + (nrows, ncols)
        # 3-D body without expert split (never produced: experts put the expert index in `lead`)
        raise ValueError(f"unexpected parameter rank for {self.key}")

    def pieces(self, a: int, b: int) -> list[_Piece]:
        """Rectangular global pieces covering local flat range [a, b) of the shard."""
        out: list[_Piece] = []
        if self.one_d:
            off, sz = self._rect(self.runs[0][2], 0, 1, a, b - a)
            return [_Piece(self.key, self.global_shape, off, sz, a, b - a)]
        C = self.C
        pos = a
        while pos < b:
            r, c = divmod(pos, C)
            run = next(x for x in self.runs if x[0] <= r < x[0] + x[1])
            lrow, nrun, lead, grow = run
            if c != 0 or b - pos < C:
                n = min(C - c, b - pos)
                off, sz = self._rect(lead, grow + (r - lrow), 1, c, n)
                out.append(_Piece(self.key, self.global_shape, off, sz, pos, n))
                pos += n
                continue
            nrows = min((b - pos) // C, lrow + nrun - r)
            off, sz = self._rect(lead, grow + (r - lrow), nrows, 0, C)
            out.append(_Piece(self.key, self.global_shape, off, sz, pos, nrows * C))
            pos += nrows * C
        return out


def _entries(model, optimizer, with_optimizer: bool):
    """(Piece, backing 1-D tensor) for every piece this rank holds."""
    out = []
    maps = {}
    for sp, _ in model.named_flat_params():
        pm = _ParamMap(model, sp)
        maps[sp.name] = (sp, pm)
        flat = model.flat_param[sp.offset:sp.offset + sp.numel]
        for pc in pm.pieces(0, sp.numel):
            out.append((pc, flat[pc.lo:pc.lo + pc.n]))
    if with_optimizer and optimizer is not None:
        for seg in optimizer.segments:
            for sp, pm in maps.values():
                a, b = max(sp.offset, seg.s_lo), min(sp.offset + sp.numel, seg.s_hi)
                if a >= b:
                    continue
                for state, buf in (("fp32_param", seg.master), ("exp_avg", seg.exp_avg),
                                   ("exp_avg_sq", seg.exp_avg_sq)):
                    src = buf[a - seg.s_lo:b - seg.s_lo]
                    for pc in pm.pieces(a - sp.offset, b - sp.offset):
                        k = f"optimizer.state.{state}.{pc.key}"
                        out.append((_Piece(k, pc.global_shape, pc.offsets, pc.sizes, pc.lo, pc.n),
                                    src[pc.lo - (a - sp.offset):pc.lo - (a - sp.offset) + pc.n]))
    return out


class _PieceSavePlanner(DefaultSavePlanner):
    def __init__(self, entries):
        super().__init__(flatten_state_dict=False)
        self._entries = entries
        self._data: dict = {}

    def create_local_plan(self) -> SavePlan:
        items = []
        for pc, t in self._entries:
            idx = MetadataIndex(pc.key, torch.Size(pc.offsets))
            self._data[(pc.key, tuple(pc.offsets))] = t.view(pc.sizes)
            items.append(WriteItem(index=idx, type=WriteItemType.SHARD, tensor_data=TensorWriteData(
                chunk=ChunkStorageMetadata(offsets=torch.Size(pc.offsets), sizes=torch.Size(pc.sizes)),
                properties=TensorProperties.create_from_tensor(t), size=torch.Size(pc.global_shape))))
        self.plan = SavePlan(items, planner_data={})
        return self.plan

    def resolve_data(self, write_item: WriteItem):
        return self._data[(write_item.index.fqn, tuple(write_item.index.offset))].detach()


class _PieceLoadPlanner(DefaultLoadPlanner):
    def __init__(self, entries):
        super().__init__()
        self._entries = entries
        self._dest: dict = {}

    def create_local_plan(self) -> LoadPlan:
        reads = []
        sdm = self.metadata.state_dict_metadata
        for pc, t in self._entries:
            if pc.key not in sdm:
                raise KeyError(f"checkpoint has no tensor {pc.key!r}")
            md = sdm[pc.key]
            if tuple(md.size) != tuple(pc.global_shape):
                raise ValueError(f"{pc.key}: checkpoint shape {tuple(md.size)} != model shape {pc.global_shape}")
            self._dest[(pc.key, tuple(pc.offsets))] = t.view(pc.sizes)
            reads += create_read_items_for_chunk_list(
                pc.key, md, [ChunkStorageMetadata(offsets=torch.Size(pc.offsets), sizes=torch.Size(pc.sizes))])
        return LoadPlan(reads)

    def lookup_tensor(self, index: MetadataIndex) -> torch.Tensor:
        return self._dest[(index.fqn, tuple(index.offset))]

    def resolve_tensor(self, read_item):
        t = self.lookup_tensor(read_item.dest_index)
        for d, (o, n) in enumerate(zip(read_item.dest_offsets, read_item.lengths)):
            t = t.narrow(d, o, n)
        return t

    def commit_tensor(self, read_item, tensor) -> None:
        pass


def _layout(model) -> dict:
    ps = model.ps
    return {"tp": ps.tp_size, "ep": ps.ep_size, "pp": ps.pp_size, "dp": ps.dp_size, "cp": ps.cp_size,
            "world_size": dist.get_world_size() if dist.is_initialized() else 1, "model": model.cfg.name}


def is_torch_dist_checkpoint(weights_dir: str) -> bool:
    it = os.path.join(weights_dir, ITER_DIR)
    return os.path.exists(os.path.join(it, "metadata.json")) and os.path.exists(os.path.join(it, ".metadata"))


_ASYNC_GROUP = None


def _async_group():
    """A gloo group over all ranks for the coordination of background saves: its
    collectives run on the save thread, apart from the training communicators."""
    global _ASYNC_GROUP
    if _ASYNC_GROUP is None:
        _ASYNC_GROUP = dist.new_group(backend="gloo")
    return _ASYNC_GROUP


def save_torch_dist(model, optimizer, weights_dir: str, save_optimizer: bool = True, async_save: bool = False):
    """Write the model (and the optimizer state) as a torch_dist checkpoint; a
    collective over the default group when it is initialised.

    ``async_save``: the pieces are first copied to pinned host memory (the only
    part the caller waits for, so training may change the weights right after),
    then planned and written by a background thread whose cross-rank
    coordination uses a separate gloo group.  Returns the write's future (its
    result is ready on every rank once rank 0's is, since rank 0 writes the
    metadata after gathering every rank's write results), or None when
    synchronous."""
    it = os.path.join(weights_dir, ITER_DIR)
    rank = dist.get_rank() if dist.is_initialized() else 0
    if rank == 0:
        os.makedirs(it, exist_ok=True)
    if dist.is_initialized():
        dist.barrier()
    fut = None
    with torch.no_grad():
        entries = _entries(model, optimizer, save_optimizer)
        if async_save:
            staged = []
            for pc, t in entries:
                host = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=t.is_cuda)
                host.copy_(t, non_blocking=True)
                staged.append((pc, host))
            if torch.cuda.is_available():
                torch.cuda.synchronize()
            fut = dcp.async_save({}, storage_writer=dcp.FileSystemWriter(it), planner=_PieceSavePlanner(staged),
                                 process_group=_async_group() if dist.is_initialized() else None,
                                 no_dist=not dist.is_initialized())
        else:
            dcp.save({}, storage_writer=dcp.FileSystemWriter(it), planner=_PieceSavePlanner(entries),
                     no_dist=not dist.is_initialized())
    if rank == 0:
        common = {"checkpoint_version": 3.0, "iteration": 0, "rl_b200_layout": _layout(model)}
        if save_optimizer and optimizer is not None:
            common["optimizer"] = {"param_groups": [{"lr": optimizer.current_lr(), "betas": (optimizer.beta1,
                                                                                          optimizer.beta2),
                                                     "eps": optimizer.eps, "weight_decay": optimizer.weight_decay}],
                                   "step": int(optimizer.step_count)}
        torch.save(common, os.path.join(it, "common.pt"))
        with open(os.path.join(it, "metadata.json"), "w") as f:
            json.dump(_METADATA, f)
        with open(os.path.join(weights_dir, "latest_checkpointed_iteration.txt"), "w") as f:
            f.write("0")
    if dist.is_initialized():
        dist.barrier()
    return fut


def load_torch_dist(model, optimizer, weights_dir: str, load_optimizer: bool = True) -> bool:
    """Fill the model (and, when the checkpoint has it, the optimizer state) from a
    torch_dist checkpoint written at any parallel layout.  Returns whether
    optimizer state was loaded."""
    it = os.path.join(weights_dir, ITER_DIR)
    reader = dcp.FileSystemReader(it)
    keys = set(reader.read_metadata().state_dict_metadata)
    has_opt = load_optimizer and optimizer is not None and any(k.startswith("optimizer.state.") for k in keys)
    with torch.no_grad():
        entries = _entries(model, optimizer, has_opt)
        dcp.load({}, storage_reader=reader, planner=_PieceLoadPlanner(entries), no_dist=not dist.is_initialized())
    if optimizer is not None:
        if has_opt:
            common = torch.load(os.path.join(it, "common.pt"), map_location="cpu", weights_only=False)
            optimizer.step_count = int((common.get("optimizer") or {}).get("step", 0))
            optimizer.restore_params_from_master()
        else:
            for seg in optimizer.segments:  # fresh moments; master follows the loaded weights
                seg.master.copy_(model.flat_param[seg.s_lo:seg.s_hi])
    return has_opt


def read_global_tensor(weights_dir: str, key: str) -> torch.Tensor:
    """One whole global tensor of a torch_dist checkpoint (single process; for
    inspection and conversion tools)."""
    it = os.path.join(weights_dir, ITER_DIR)
    md = dcp.FileSystemReader(it).read_metadata().state_dict_metadata[key]
    out = torch.empty(tuple(md.size), dtype=md.properties.dtype)
    dcp.load({key: out}, storage_reader=dcp.FileSystemReader(it), no_dist=True)
    return out
