"""GEMM entry points used by every linear layer.

Three shapes of product cover a linear layer's forward and backward passes
(all row-major, ``W [N, K]``):

* ``mm_nt(a [M,K], b [N,K]) = a @ b^T``  (forward),
* ``mm_nn(a [M,N], b [N,K]) = a @ b``    (input gradient),
* ``mm_tn(a [M,N], b [M,K]) = a^T @ b``  (weight gradient; ``mm_tn_accumulate``
  adds it into an fp32 buffer).

On CUDA, ``mm_nt`` runs the hand-written tcgen05 kernel of ``csrc/gemm_tcgen05.cu``
(TMA-fed shared-memory stages, ``tcgen05.mma`` with the accumulator in tensor
memory, persistent tile loop) when the shape is tile-aligned; the other
products and unaligned shapes use the library GEMM (cuBLAS through
``torch.matmul``), which is the plain-GEMM baseline.
"""

from __future__ import annotations

import os

import torch

from rl_b200.ops._ext import ext, has_ext, use_native

__all__ = ["mm_nt", "mm_nn", "mm_tn", "mm_tn_accumulate", "native_gemm_supported"]

_NATIVE_GEMM = os.environ.get("RL_B200_NATIVE_GEMM", "1") == "1"


def native_gemm_supported(M: int, N: int, K: int, dtype) -> bool:
    return (
        _NATIVE_GEMM and dtype == torch.bfloat16 and has_ext() and hasattr(ext(), "gemm_nt")
        and K % 64 == 0 and N % 16 == 0 and M > 0
    )


def mm_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if use_native(a) and native_gemm_supported(a.shape[0], b.shape[0], a.shape[1], a.dtype) \
            and a.is_contiguous() and b.is_contiguous():
        return ext().gemm_nt(a, b)
    return torch.matmul(a, b.t())


def mm_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.matmul(a, b)


def mm_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.matmul(a.t(), b)


def mm_tn_accumulate(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> None:
    """``out += a^T @ b`` with fp32 ``out``."""
    if a.is_cuda:
        out.add_(torch.mm(a.t(), b, out_dtype=torch.float32))
    else:
        out.add_(torch.matmul(a.t().float(), b.float()))
