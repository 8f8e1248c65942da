"""Grouped (per-expert) GEMM for MoE layers (native component N11).

``grouped_mm_nt(x [N, K], w [E, M, K], counts [E]) -> y [N, M]`` where rows
``[off_e, off_e + counts[e])`` of ``x`` are multiplied by ``w[e]^T``.  Backward:
``dx`` is the grouped ``dy @ w[e]`` and ``dw[e] = dy_e^T @ x_e`` (accumulated into
``w.main_grad`` when present, like ``rl_b200.ops.linear``).

CUDA path: the forward runs the tcgen05 grouped kernel of ``csrc/gemm_grouped.cu``
(tile schedule built on the device from the offsets) when
``RL_B200_NATIVE_GROUPED=1``, else the library's ragged grouped GEMM
(``torch._grouped_mm``), which also takes the input gradient; weight gradients
are per-expert GEMMs.  The CPU path loops over experts in fp32.
"""

from __future__ import annotations

import os

import torch

__all__ = ["grouped_mm_nt"]

_NATIVE = os.environ.get("RL_B200_NATIVE_GROUPED", "0") == "1"


def _native_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    from rl_b200.ops._ext import has_ext

    return (_NATIVE and x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and has_ext()
            and x.shape[1] % 64 == 0 and w.shape[1] % 128 == 0 and w.shape[0] <= 512)


def _offsets(counts: torch.Tensor) -> torch.Tensor:
    return torch.cumsum(counts.to(torch.int32), 0).to(torch.int32)


def _loop_nt(x, w, counts):
    out = x.new_empty(x.shape[0], w.shape[1])
    start = 0
    for e, c in enumerate(counts.tolist()):
        if c:
            out[start:start + c] = torch.matmul(x[start:start + c], w[e].t())
        start += c
    return out


def _loop_nn(dy, w, counts):
    out = dy.new_empty(dy.shape[0], w.shape[2])
    start = 0
    for e, c in enumerate(counts.tolist()):
        if c:
            out[start:start + c] = torch.matmul(dy[start:start + c], w[e])
        start += c
    return out


def _gmm_ok(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and hasattr(torch, "_grouped_mm")


class _GroupedNT(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, counts):
        ctx.save_for_backward(x, w, counts)
        if x.shape[0] == 0:
            return x.new_zeros(0, w.shape[1])
        if _native_ok(x, w):
            from rl_b200.ops._ext import ext

            return ext().grouped_gemm_nt(x.contiguous(), w.contiguous(), _offsets(counts))
        if _gmm_ok(x):
            return torch._grouped_mm(x, w.transpose(1, 2), offs=_offsets(counts))
        return _loop_nt(x, w, counts)

    @staticmethod
    def backward(ctx, dy):
        x, w, counts = ctx.saved_tensors
        dy = dy.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            if x.shape[0] == 0:
                dx = torch.zeros_like(x)
            elif _gmm_ok(x):
                dx = torch._grouped_mm(dy, w, offs=_offsets(counts))
            else:
                dx = _loop_nn(dy, w, counts)
        dw = None
        if ctx.needs_input_grad[1]:
            main = getattr(w, "main_grad", None)
            acc = main if main is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
            start = 0
            for e, c in enumerate(counts.tolist()):
                if c:
                    a, b = dy[start:start + c], x[start:start + c]
                    if a.is_cuda:
                        acc[e].add_(torch.mm(a.t(), b, out_dtype=torch.float32))
                    else:
                        acc[e].add_(torch.matmul(a.t().float(), b.float()))
                start += c
            dw = None if main is not None else acc.to(w.dtype)
        return dx, dw, None


def grouped_mm_nt(x: torch.Tensor, w: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    return _GroupedNT.apply(x, w, counts)
