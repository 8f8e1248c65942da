"""GEMM entry points used by every linear layer.

Three shapes of product cover a linear layer's forward and backward passes
(all row-major, ``W [N, K]``):

* ``mm_nt(a [M,K], b [N,K]) = a @ b^T``  (forward),
* ``mm_nn(a [M,N], b [N,K]) = a @ b``    (input gradient),
* ``mm_tn(a [M,N], b [M,K]) = a^T @ b``  (weight gradient; ``mm_tn_accumulate``
  adds it into an fp32 buffer).

On CUDA all three run the hand-written tcgen05 kernel of ``csrc/gemm_sm100.cu``
(TMA-fed shared-memory stages, ``tcgen05.mma`` with the accumulator in tensor
memory, persistent tile loop; 2-CTA 256x256 tiles when the product fills the
GPU, else 1-CTA 128x256): the input gradient reads ``W`` as an MN-major
operand and the weight gradient reads both ``dy`` and ``x`` as MN-major
operands, so nothing is transposed in memory, and the weight gradient is added
into the fp32 main-grad buffer by the kernel's epilogue.  Decode-shaped
products (a few rows) stream the weight in ``csrc/gemm_decode.cu``.  Shapes the
kernels cannot take (a contiguous dimension that is not a multiple of 8, or too
few output tiles to occupy the SMs) use the library GEMM (cuBLAS through
``torch.matmul``), the plain-GEMM baseline.

Reference: Transformer Engine's cuBLASLt GEMMs behind Megatron-core linear
layers (``nemo_rl/models/megatron/setup.py:2520``).
"""

from __future__ import annotations

import os

import torch

from rl_b200.ops._ext import ext, has_ext, use_native

__all__ = ["mm_nt", "mm_nn", "mm_tn", "mm_tn_accumulate", "native_gemm_supported", "decode_gemm_supported"]

_NATIVE_GEMM = os.environ.get("RL_B200_NATIVE_GEMM", "1") == "1"
# RL_B200_DECODE_GEMM=0 sends decode-shaped products to the library GEMM (A/B timing)
_DECODE_GEMM = os.environ.get("RL_B200_DECODE_GEMM", "1") == "1"
# fixed K split of the decode kernel (0 = chosen per shape); 1 accumulates K in the
# same order as the large-tile kernel (numerics studies)
_DECODE_SPLITS = int(os.environ.get("RL_B200_DECODE_SPLITS", "0"))


_NUM_SMS = None


def _sms() -> int:
    global _NUM_SMS
    if _NUM_SMS is None:
        _NUM_SMS = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count \
            if torch.cuda.is_available() else 148
    return _NUM_SMS


def native_gemm_supported(M: int, N: int, K: int, dtype, inner: tuple = ()) -> bool:
    """Whether the tcgen05 kernel takes an ``M x N`` output reducing over ``K``.

    It computes 128 x 256 (or 256 x 256) output tiles, one CTA (pair) per SM
    (pair); shapes that give fewer tiles than half the SMs (decode-time GEMMs
    with a handful of rows) leave most of the GPU idle in it.  ``inner`` lists
    the contiguous (last) dimension of every operand, which TMA needs as a
    multiple of 8 elements (16-byte rows)."""
    if not (_NATIVE_GEMM and dtype == torch.bfloat16 and has_ext() and M > 0 and N > 0 and K > 0):
        return False
    if any(d % 8 for d in inner):
        return False
    tiles = -(-M // 128) * -(-N // 256)
    return tiles * 2 >= _sms()


def decode_gemm_supported(M: int, N: int, K: int, dtype) -> bool:
    """Few-row products (rollout decode: one token per sequence) stream the
    weight matrix: the split-K transposed tcgen05 kernel of ``csrc/gemm_decode.cu``."""
    return (_DECODE_GEMM and dtype == torch.bfloat16 and has_ext() and 0 < M <= 256 and N >= 128
            and K % 8 == 0)


# Up to this many rows a product streams its weight (memory-bound on B200: the
# bf16 ridge point is ~250 FLOP per weight byte, i.e. ~125 rows), so the
# decode-shaped kernel is used whatever N is.
DECODE_MAX_ROWS = 128


def mm_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M,K] @ b[N,K]^T``."""
    if use_native(a) and a.is_contiguous() and b.is_contiguous() and b.dtype == a.dtype:
        M, N, K = a.shape[0], b.shape[0], a.shape[1]
        if M <= DECODE_MAX_ROWS and decode_gemm_supported(M, N, K, a.dtype):
            if _DECODE_SPLITS:
                return ext().gemm_decode_split(a, b, _DECODE_SPLITS)
            return ext().gemm_decode(a, b)
        if native_gemm_supported(M, N, K, a.dtype, (K,)):
            out = torch.empty(M, N, device=a.device, dtype=a.dtype)
            ext().gemm_sm100(a, b, out, False, False, False, 0)
            return out
        if decode_gemm_supported(M, N, K, a.dtype):
            return ext().gemm_decode(a, b)
    return torch.matmul(a, b.t())


def mm_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M,N] @ b [N,K]`` (input gradient: ``b`` is the weight, read MN-major)."""
    if use_native(a) and a.is_contiguous() and b.is_contiguous() and b.dtype == a.dtype:
        M, Nr, K = a.shape[0], a.shape[1], b.shape[1]
        if native_gemm_supported(M, K, Nr, a.dtype, (Nr, K)):
            out = torch.empty(M, K, device=a.device, dtype=a.dtype)
            ext().gemm_sm100(a, b, out, False, True, False, 0)
            return out
    return torch.matmul(a, b)


def mm_tn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a [M,N]^T @ b [M,K]`` -> ``[N, K]`` (weight gradient; both operands MN-major)."""
    if use_native(a) and a.is_contiguous() and b.is_contiguous() and b.dtype == a.dtype:
        Mr, N, K = a.shape[0], a.shape[1], b.shape[1]
        if native_gemm_supported(N, K, Mr, a.dtype, (N, K)):
            out = torch.empty(N, K, device=a.device, dtype=a.dtype)
            ext().gemm_sm100(a, b, out, True, True, False, 0)
            return out
    return torch.matmul(a.t(), b)


def mm_tn_accumulate(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> None:
    """``out += a^T @ b`` with fp32 ``out`` (the weight gradient added into main-grad
    by the GEMM epilogue)."""
    if a.is_cuda:
        if (use_native(a) and a.is_contiguous() and b.is_contiguous() and out.is_contiguous()
                and out.dtype == torch.float32 and b.dtype == a.dtype):
            Mr, N, K = a.shape[0], a.shape[1], b.shape[1]
            if native_gemm_supported(N, K, Mr, a.dtype, (N, K)):
                ext().gemm_sm100(a, b, out, True, True, True, 0)
                return
        out.add_(torch.mm(a.t(), b, out_dtype=torch.float32))
    else:
        out.add_(torch.matmul(a.t().float(), b.float()))
