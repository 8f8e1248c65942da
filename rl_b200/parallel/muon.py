"""Muon: momentum orthogonalised by Newton-Schulz, for the 2-D weights of the
linear layers (``megatron_cfg.optimizer.optimizer: dist_muon``).

For a weight ``W`` with gradient ``G`` (after clipping):

    M <- M + (1 - mu) (G - M)                  (momentum, EMA form)
    U  = G + mu (M - G) if nesterov else M
    O  = NS5(U)                                (approximately U V^T of U's SVD)
    W <- W (1 - lr wd) - lr * scale(out, in) * extra_scale_factor * O

``NS5`` is the quintic Newton-Schulz iteration of Jordan et al. ("Muon: An
optimizer for hidden layers in neural networks", 2024): ``X = U / |U|_F``,
then ``steps`` times ``X <- a X + (b A + c A^2) X`` with ``A = X X^T`` and
``(a, b, c) = (3.4445, -4.7750, 2.0315)``.  Because ``p(X X^T) X = X p(X^T X)``
the iteration can run from either side: the row-split shards of a
tensor-parallel matrix update with the small ``X^T X`` Gram summed over the
TP group, the column-split ones with ``X X^T`` - the ``distributed`` mode,
identical to orthogonalising the full matrix.  ``duplicated`` all-gathers the
full matrix and keeps this rank's slice; ``blockwise`` orthogonalises each
rank's shard on its own (no communication; a different update).

``scale_mode`` (``muon_scale_mode``): ``spectral`` ``sqrt(max(out, in))``
(with ``extra_scale_factor`` 0.2 the update RMS matches AdamW's: Liu et al.,
"Muon is Scalable for LLM Training", arXiv:2502.16982), ``shape_scaling``
``sqrt(max(1, out / in))`` (Jordan et al.), ``unit_rms_norm``
``sqrt(out / in)`` (Pethick et al., "Training Deep Learning Models with Norm-
Constrained LMOs", arXiv:2502.07529).  ``split_qkv`` orthogonalises the q, k
and v rows of the fused projection separately.  Embeddings, the LM head,
the MoE router, norms and biases keep AdamW.

Reference: ``docs/guides/muon-optimizer.md`` (the Megatron optimizer options
``muon_momentum``, ``muon_nesterov``, ``muon_scale_mode``,
``muon_fp32_matmul_prec``, ``muon_num_ns_steps``, ``muon_tp_mode``,
``muon_extra_scale_factor``, ``muon_split_qkv``).
"""

from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

__all__ = ["MuonConfig", "newton_schulz", "orthogonalize", "muon_scale", "is_muon_param"]

NS_COEFFS = (3.4445, -4.7750, 2.0315)
_MUON_SUFFIXES = ("self_attn.qkv_proj.weight", "self_attn.o_proj.weight", "mlp.gate_up_proj.weight",
                  "mlp.down_proj.weight", "mlp.experts.gate_up_proj", "mlp.experts.down_proj")


@dataclass
class MuonConfig:
    momentum: float = 0.95
    nesterov: bool = False
    scale_mode: str = "spectral"
    fp32_matmul_prec: str = "medium"
    num_ns_steps: int = 5
    tp_mode: str = "blockwise"
    extra_scale_factor: float = 1.0
    split_qkv: bool = True
    eps: float = 1e-7

    @classmethod
    def from_megatron(cls, mopt: dict) -> Optional["MuonConfig"]:
        """``None`` unless ``optimizer`` names Muon."""
        if str(mopt.get("optimizer", "adam")).lower() not in ("muon", "dist_muon"):
            return None
        c = cls(momentum=float(mopt.get("muon_momentum", 0.95)), nesterov=bool(mopt.get("muon_nesterov", False)),
                scale_mode=str(mopt.get("muon_scale_mode", "spectral")),
                fp32_matmul_prec=str(mopt.get("muon_fp32_matmul_prec", "medium")),
                num_ns_steps=int(mopt.get("muon_num_ns_steps", 5)), tp_mode=str(mopt.get("muon_tp_mode", "blockwise")),
                extra_scale_factor=float(mopt.get("muon_extra_scale_factor", 1.0)),
                split_qkv=bool(mopt.get("muon_split_qkv", True)))
        if c.scale_mode not in ("spectral", "shape_scaling", "unit_rms_norm"):
            raise ValueError(f"muon_scale_mode {c.scale_mode!r}: expected spectral, shape_scaling or unit_rms_norm")
        if c.tp_mode not in ("blockwise", "duplicated", "distributed"):
            raise ValueError(f"muon_tp_mode {c.tp_mode!r}: expected blockwise, duplicated or distributed")
        if c.fp32_matmul_prec not in ("medium", "high", "highest"):
            raise ValueError(f"muon_fp32_matmul_prec {c.fp32_matmul_prec!r}: expected medium, high or highest")
        if not 0.0 <= c.momentum < 1.0 or c.num_ns_steps < 1:
            raise ValueError("muon_momentum must lie in [0, 1) and muon_num_ns_steps be >= 1")
        return c


def is_muon_param(name: str) -> bool:
    return name.endswith(_MUON_SUFFIXES)


def muon_scale(out_dim: int, in_dim: int, mode: str) -> float:
    if mode == "spectral":
        return math.sqrt(max(out_dim, in_dim))
    if mode == "shape_scaling":
        return math.sqrt(max(1.0, out_dim / in_dim))
    return math.sqrt(out_dim / in_dim)


@contextlib.contextmanager
def _matmul_precision(prec: str):
    old = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision(prec)
    try:
        yield
    finally:
        torch.set_float32_matmul_precision(old)


def newton_schulz(u: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """NS5 of ``u`` (``[..., m, n]``, batched over leading dims) in fp32."""
    a, b, c = NS_COEFFS
    x = u.float()
    tall = x.shape[-2] > x.shape[-1]
    if tall:
        x = x.transpose(-2, -1)
    x = x / x.flatten(-2).norm(dim=-1).clamp_min(eps)[..., None, None]
    for _ in range(steps):
        A = x @ x.transpose(-2, -1)
        x = a * x + (b * A + c * (A @ A)) @ x
    return x.transpose(-2, -1) if tall else x


def _ns_distributed(u: torch.Tensor, split_dim: int, steps: int, eps: float, group) -> torch.Tensor:
    """NS5 of the matrix whose shards along ``split_dim`` (-2: rows, -1:
    columns) the TP group holds; every step all-reduces one Gram matrix of
    the unsplit side."""
    a, b, c = NS_COEFFS
    x = u.float()
    sq = (x * x).flatten(-2).sum(-1)
    dist.all_reduce(sq, group=group)
    x = x / sq.sqrt().clamp_min(eps)[..., None, None]
    for _ in range(steps):
        if split_dim == -2:  # rows split: X <- a X + X (b B + c B^2), B = X^T X summed over shards
            B = x.transpose(-2, -1) @ x
            dist.all_reduce(B, group=group)
            x = a * x + x @ (b * B + c * (B @ B))
        else:  # columns split: X <- a X + (b A + c A^2) X, A = X X^T summed over shards
            A = x @ x.transpose(-2, -1)
            dist.all_reduce(A, group=group)
            x = a * x + (b * A + c * (A @ A)) @ x
    return x


def orthogonalize(u: torch.Tensor, tp_dim: Optional[int], cfg: MuonConfig, tp_group=None) -> tuple[torch.Tensor, tuple]:
    """Orthogonalised update of one (local) matrix block and the (out, in)
    shape its scale is computed from.  ``tp_dim`` is the sharded dim counted
    from the end (-2 rows, -1 columns) or ``None``."""
    tp = dist.get_world_size(tp_group) if (tp_group is not None and dist.is_initialized()) else 1
    out_dim, in_dim = u.shape[-2], u.shape[-1]
    with _matmul_precision(cfg.fp32_matmul_prec):
        if tp_dim is None or tp == 1 or cfg.tp_mode == "blockwise":
            return newton_schulz(u, cfg.num_ns_steps, cfg.eps), (out_dim, in_dim)
        full_shape = (out_dim * tp, in_dim) if tp_dim == -2 else (out_dim, in_dim * tp)
        if cfg.tp_mode == "distributed":
            return _ns_distributed(u, tp_dim, cfg.num_ns_steps, cfg.eps, tp_group), full_shape
        parts = [torch.empty_like(u, dtype=torch.float32) for _ in range(tp)]
        dist.all_gather(parts, u.float().contiguous(), group=tp_group)
        o = newton_schulz(torch.cat(parts, dim=tp_dim), cfg.num_ns_steps, cfg.eps)
        r = dist.get_rank(tp_group)
        return o.narrow(tp_dim, r * u.shape[tp_dim], u.shape[tp_dim]), full_shape
