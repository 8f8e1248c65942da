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

__all__ = ["mm_nt", "mm_nn", "mm_tn", "mm_tn_accumulate", "native_gemm_supported", "decode_gemm_supported"]

_NATIVE_GEMM = os.environ.get("RL_B200_NATIVE_GEMM", "1") == "1"
# the decode-shaped kernel is opt-in until it beats the library GEMM on every decode shape
_DECODE_GEMM = os.environ.get("RL_B200_DECODE_GEMM", "0") == "1"


_NUM_SMS = None


def _sms() -> int:
    global _NUM_SMS
    if _NUM_SMS is None:
        _NUM_SMS = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count \
            if torch.cuda.is_available() else 148
    return _NUM_SMS


def native_gemm_supported(M: int, N: int, K: int, dtype) -> bool:
    """The persistent tcgen05 kernel computes 128 x 256 output tiles, one CTA per
    SM; shapes that give fewer tiles than half the SMs (decode-time GEMMs with a
    handful of rows) leave most of the GPU idle in it, so they go to the library
    GEMM's split-K kernels instead."""
    if not (_NATIVE_GEMM and dtype == torch.bfloat16 and has_ext() and K % 64 == 0 and N % 16 == 0 and M > 0):
        return False
    bn = 256 if N >= 256 else 128
    tiles = -(-M // 128) * -(-N // bn)
    return tiles * 2 >= _sms()


def decode_gemm_supported(M: int, N: int, K: int, dtype) -> bool:
    """Few-row products (rollout decode: one token per sequence) stream the
    weight matrix: the split-K transposed tcgen05 kernel of ``csrc/gemm_decode.cu``."""
    return (_DECODE_GEMM and dtype == torch.bfloat16 and has_ext() and 0 < M <= 256 and N >= 128
            and K % 8 == 0)


def mm_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if use_native(a) and a.is_contiguous() and b.is_contiguous():
        M, N, K = a.shape[0], b.shape[0], a.shape[1]
        if native_gemm_supported(M, N, K, a.dtype):
            return ext().gemm_nt(a, b)
        if decode_gemm_supported(M, N, K, a.dtype):
            return ext().gemm_decode(a, b)
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
