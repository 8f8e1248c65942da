"""Train-layout -> generation-layout weight reshard plans.

The training model of a tensor-parallel group of ``t`` ranks holds shard ``i``
of every TP-sharded weight (rows for column-parallel weights - with the fused
``[q | k | v]`` and ``[gate | up]`` row sections split section by section -
columns for row-parallel ones).  A generation model of TP ``g`` (``g`` divides
``t``) on the same GPU needs shard ``j = tp_rank % g`` of the generation
layout, i.e. the training shards ``[j*t/g, (j+1)*t/g)`` of every section,
placed side by side.

``build_tasks`` turns that into 2-D copy regions between the training ranks'
flat parameter buffers and the generation model's flat buffer; ``quant_tasks``
cuts the regions of the linear weights into the 128 x 128 blocks of an e4m3
block-scaled copy.  The same task tables drive the native kernels
(``csrc/refit.cu``, which load the peers' shards over NVLink) and the torch
reference ``apply_tasks_reference`` used on CPU.

Reference: ``nccl_reshard_utils.py`` placement rules (``MeshInfo``) and the
striped receive + all-gather of ``weight_sync/xferdtensor_python.py:642-668``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

__all__ = ["Region", "build_regions", "copy_tasks", "quant_tasks", "apply_regions_reference",
           "quant_regions_reference", "QUANT_SUFFIXES"]

# linear weights that the fp8 rollout quantises (embeddings, norms, LM head stay bf16)
QUANT_SUFFIXES = ("qkv_proj.weight", "o_proj.weight", "gate_up_proj.weight", "down_proj.weight")


@dataclass
class Region:
    """rows x cols elements: source rank / offset / leading dim -> destination
    offset / leading dim (elements of the flat buffers), plus where the region
    sits inside its destination parameter (for block quantisation)."""
    name: str
    src_rank: int
    src_off: int
    src_ld: int
    dst_off: int
    dst_ld: int
    rows: int
    cols: int
    dst_row0: int      # region's first row / col inside the destination parameter
    dst_col0: int
    param_rows: int    # destination parameter shape (2-D view)
    param_cols: int
    param_off: int     # destination parameter offset in the flat buffer


def _sections(name: str, cfg, full_rows: int) -> list[int]:
    if name.endswith("qkv_proj.weight"):
        hd = cfg.head_dim
        return [cfg.num_heads * hd, cfg.num_kv_heads * hd, cfg.num_kv_heads * hd]
    if name.endswith("gate_up_proj.weight"):
        return [full_rows // 2, full_rows // 2]
    return [full_rows]


def build_regions(train_specs, gen_specs, cfg, t: int, g: int, tp_rank: int) -> list[Region]:
    """Copy regions that assemble generation shard ``tp_rank % g`` (of TP ``g``)
    from the ``t`` training shards.  Replicated parameters come from the local
    training rank ``tp_rank``."""
    if t % g:
        raise ValueError(f"generation TP {g} must divide training TP {t}")
    if any(sp.ep_dim is not None for sp in train_specs):
        raise NotImplementedError("expert-parallel weights keep their layout (generation EP = training EP)")
    tmap = {sp.name: sp for sp in train_specs}
    j = tp_rank % g
    per = t // g
    out: list[Region] = []
    for gs in gen_specs:
        ts = tmap[gs.name]
        shape = gs.shape if len(gs.shape) == 2 else (1, gs.numel)
        R, C = shape
        tshape = ts.shape if len(ts.shape) == 2 else (1, ts.numel)
        if gs.tp_dim is None or t == 1:
            out.append(Region(gs.name, tp_rank, ts.offset, tshape[1], gs.offset, C, R, C, 0, 0, R, C, gs.offset))
            continue
        if gs.tp_dim is not None and len(gs.shape) != 2:
            raise NotImplementedError(f"{gs.name}: a tensor-parallel 1-D parameter (attention bias) needs the "
                                      "rollout TP to equal the training TP")
        if gs.tp_dim == 0:
            full_rows = tshape[0] * t
            sec = _sections(gs.name, cfg, full_rows)
            t_row, g_row = 0, 0
            for L in sec:
                lt, lg = L // t, L // g
                for k in range(per):
                    i = j * per + k
                    out.append(Region(gs.name, i, ts.offset + t_row * C, C, gs.offset + (g_row + k * lt) * C, C,
                                      lt, C, g_row + k * lt, 0, R, C, gs.offset))
                t_row += lt
                g_row += lg
        elif gs.tp_dim == 1:
            ct = tshape[1]
            for k in range(per):
                i = j * per + k
                out.append(Region(gs.name, i, ts.offset, ct, gs.offset + k * ct, C, R, ct, 0, k * ct, R, C, gs.offset))
        else:
            raise ValueError(f"unsupported tp_dim {gs.tp_dim} for {gs.name}")
    return out


def _addr(r: Region, src_ptrs, elt: int) -> int:
    return int(src_ptrs[r.src_rank]) + r.src_off * elt


def copy_tasks(regions: list[Region], src_ptrs, max_elems: int = 32768, elt: int = 2) -> np.ndarray:
    """int64 [n, 8] task table of the bf16 copy kernel: every region cut into
    row chunks of at most ``max_elems`` elements."""
    rows = []
    for r in regions:
        if r.cols % 8 or r.src_ld % 8 or r.dst_ld % 8 or r.src_off % 8 or r.dst_off % 8:
            raise ValueError(f"{r.name}: regions must be 16-byte aligned (multiples of 8 elements)")
        step = max(1, max_elems // r.cols)
        base = _addr(r, src_ptrs, elt)
        for r0 in range(0, r.rows, step):
            n = min(step, r.rows - r0)
            rows.append((base + r0 * r.src_ld * elt, r.src_ld, r.dst_off + r0 * r.dst_ld, r.dst_ld, n, r.cols, 0, 0))
    return np.asarray(rows, dtype=np.int64).reshape(-1, 8)


def quant_layout(gen_specs, block: int = 128):
    """Byte offsets of every quantised parameter in the e4m3 buffer and of its
    ``[ceil(R/b), ceil(C/b)]`` fp32 scales; returns (layout, q_bytes, n_scales)."""
    lay, qoff, soff = {}, 0, 0
    for gs in gen_specs:
        if not gs.name.endswith(QUANT_SUFFIXES):
            continue
        R, C = gs.shape
        nb, kb = -(-R // block), -(-C // block)
        lay[gs.name] = (qoff, soff, R, C, nb, kb)
        qoff += -(-(R * C) // 16) * 16
        soff += nb * kb
    return lay, qoff, soff


def quant_tasks(regions: list[Region], layout: dict, src_ptrs, block: int = 128, elt: int = 2) -> np.ndarray:
    """int64 [n, 8] task table of the quantising kernel: one task per
    ``block x block`` tile of each quantised destination weight; every tile
    must come from ONE region (training shard boundaries on block multiples)."""
    rows = []
    for r in regions:
        if r.name not in layout:
            continue
        qoff, soff, R, C, nb, kb = layout[r.name]
        if r.dst_row0 % block or r.dst_col0 % block or (r.rows % block and r.dst_row0 + r.rows != R) \
                or (r.cols % block and r.dst_col0 + r.cols != C):
            raise ValueError(f"{r.name}: shard boundaries are not multiples of the {block}-block")
        base = _addr(r, src_ptrs, elt)
        for br in range(0, r.rows, block):
            for bc in range(0, r.cols, block):
                gr, gc = r.dst_row0 + br, r.dst_col0 + bc
                rows.append((base + (br * r.src_ld + bc) * elt, r.src_ld, qoff + gr * C + gc, C,
                             min(block, r.rows - br), min(block, r.cols - bc),
                             soff + (gr // block) * kb + gc // block, 0))
    return np.asarray(rows, dtype=np.int64).reshape(-1, 8)


# ------------------------------------------------------------- torch reference
def apply_regions_reference(regions: list[Region], srcs: list[torch.Tensor], dst: torch.Tensor) -> None:
    """What the copy kernel does, with torch indexing (CPU tests / fallback)."""
    for r in regions:
        s = srcs[r.src_rank]
        src = s[r.src_off: r.src_off + (r.rows - 1) * r.src_ld + r.cols].as_strided((r.rows, r.cols), (r.src_ld, 1))
        d = dst[r.dst_off: r.dst_off + (r.rows - 1) * r.dst_ld + r.cols].as_strided((r.rows, r.cols), (r.dst_ld, 1))
        d.copy_(src)


def quant_regions_reference(gen_flat: torch.Tensor, layout: dict, q: torch.Tensor, scales: torch.Tensor,
                            gen_specs, pow2: bool = False, block: int = 128) -> None:
    """Quantise the (already resharded) generation weights block-wise."""
    from rl_b200.ops.quant import quant_fp8_block_ref

    spec = {gs.name: gs for gs in gen_specs}
    for name, (qoff, soff, R, C, nb, kb) in layout.items():
        w = gen_flat[spec[name].offset: spec[name].offset + R * C].view(R, C)
        qq, ss = quant_fp8_block_ref(w, block, pow2)
        q[qoff: qoff + R * C].copy_(qq.view(-1).view(torch.uint8))
        scales[soff: soff + nb * kb].copy_(ss.reshape(-1))
