"""Quantisation-aware training (fake quantisation with a straight-through estimator).

``policy.quant_cfg`` selects the format the policy is trained to tolerate:

* ``"FP8_BLOCK_CFG"``   - weights in 128 x 128 e4m3 blocks, inputs 1 x 128 e4m3
  (what the fp8 rollout executes, so training sees the rollout's numerics);
* ``"FP8_DEFAULT_CFG"`` - per-tensor e4m3 weights and inputs (calibrated input amax);
* ``"NVFP4_DEFAULT_CFG"`` / ``"NVFP4_W4A16_CFG"`` - e2m1 values in 16-element blocks
  with e4m3 block scales under a per-tensor fp32 scale (weights and inputs, or
  weights only);
* a dict ``{"weight": {"format", "block"}, "input": {...} | None, "ignore": [glob, ...]}``.

The linear layers of the training forward apply ``x + (q(x) - x).detach()`` to
their weights and inputs (gradients pass straight through).  ``calibrate``
runs forwards that record the per-layer input amax used by per-tensor input
quantisers; ``quantizer_stats`` reports them.  The LM head, embeddings, norms
and MoE routers are never quantised (the reference's default ignore list).

Reference: the ModelOpt quantised policy worker
(``nemo_rl/modelopt/models/policy/workers/megatron_quant_policy_worker.py:195``
``_quantize``, ``:409`` ``get_quantizer_stats``; ignore patterns
``nemo_rl/modelopt/utils.py`` ``DEFAULT_NVFP4_IGNORE``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from fnmatch import fnmatchcase
from typing import Optional

import torch

__all__ = ["QuantSpec", "QATConfig", "QAT", "fake_quant", "E2M1_VALUES"]

FP8_MAX = 448.0
E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
_DEFAULT_IGNORE = ["lm_head*", "*embed_tokens*", "*mlp.gate.weight", "*router*", "score*"]


@dataclass
class QuantSpec:
    fmt: str                    # "fp8" | "nvfp4"
    block: Optional[tuple] = None  # fp8: (rows, cols) block or None (per tensor); nvfp4: 16-wide


@dataclass
class QATConfig:
    weight: Optional[QuantSpec]
    input: Optional[QuantSpec]
    ignore: list = field(default_factory=lambda: list(_DEFAULT_IGNORE))

    @staticmethod
    def from_cfg(cfg) -> Optional["QATConfig"]:
        if cfg is None or cfg is False:
            return None
        presets = {
            "FP8_BLOCK_CFG": (QuantSpec("fp8", (128, 128)), QuantSpec("fp8", (1, 128))),
            "FP8_DEFAULT_CFG": (QuantSpec("fp8"), QuantSpec("fp8")),
            "NVFP4_DEFAULT_CFG": (QuantSpec("nvfp4", (1, 16)), QuantSpec("nvfp4", (1, 16))),
            "NVFP4_W4A16_CFG": (QuantSpec("nvfp4", (1, 16)), None),
        }
        if isinstance(cfg, str):
            if cfg not in presets:
                raise ValueError(f"unknown quant_cfg preset {cfg!r}; known: {sorted(presets)}")
            w, i = presets[cfg]
            return QATConfig(w, i)

        def spec(d):
            if not d:
                return None
            b = d.get("block")
            return QuantSpec(str(d["format"]).lower(), tuple(b) if b is not None else None)

        return QATConfig(spec(cfg.get("weight")), spec(cfg.get("input")), list(cfg.get("ignore", _DEFAULT_IGNORE)))


# ----------------------------------------------------------------- fake quant
def _fp8_round(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).float()


def _blocks(x: torch.Tensor, br: int, bc: int):
    R, C = x.shape
    pr, pc = (-R) % br, (-C) % bc
    xp = torch.nn.functional.pad(x, (0, pc, 0, pr))
    return xp.view((R + pr) // br, br, (C + pc) // bc, bc), R, C


def _fq_fp8(x: torch.Tensor, block, amax: Optional[torch.Tensor]) -> torch.Tensor:
    xf = x.float().reshape(-1, x.shape[-1])
    if block is None:
        a = amax if amax is not None else xf.abs().amax()
        s = a.clamp_min(1e-12) / FP8_MAX
        return (_fp8_round(xf / s) * s).view(x.shape)
    b, R, C = _blocks(xf, *block)
    s = b.abs().amax(dim=(1, 3), keepdim=True).clamp_min(1e-12) / FP8_MAX
    q = _fp8_round(b / s) * s
    return q.reshape(b.shape[0] * b.shape[1], -1)[:R, :C].reshape(x.shape)


def _e2m1_round(v: torch.Tensor) -> torch.Tensor:
    """Round to the nearest e2m1 value (|v| <= 6), ties to the larger magnitude."""
    grid = E2M1_VALUES.to(v.device)
    a = v.abs().clamp(max=6.0)
    idx = torch.bucketize(a, (grid[1:] + grid[:-1]) / 2)
    return grid[idx] * v.sign()


def _fq_nvfp4(x: torch.Tensor, amax: Optional[torch.Tensor]) -> torch.Tensor:
    """16-element blocks, e4m3 block scales, fp32 per-tensor scale so that the
    largest block scale is 448 (the NVFP4 two-level scaling)."""
    xf = x.float().reshape(-1, x.shape[-1])
    a = amax if amax is not None else xf.abs().amax()
    g = a.clamp_min(1e-12) / (6.0 * FP8_MAX)
    b, R, C = _blocks(xf, 1, 16)
    bs = b.abs().amax(dim=3, keepdim=True) / 6.0
    bs = _fp8_round(bs / g) * g                     # block scale stored in e4m3
    q = _e2m1_round(b / bs.clamp_min(1e-30)) * bs
    return q.reshape(b.shape[0], -1)[:R, :C].reshape(x.shape)


def fake_quant(x: torch.Tensor, spec: QuantSpec, amax: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Quantise-dequantise ``x`` (returned in x's dtype)."""
    if spec.fmt == "fp8":
        y = _fq_fp8(x, spec.block, amax)
    elif spec.fmt == "nvfp4":
        y = _fq_nvfp4(x, amax)
    else:
        raise ValueError(f"unsupported quantisation format {spec.fmt!r}")
    return y.to(x.dtype)


class QAT:
    """Per-layer quantisers of one model."""

    def __init__(self, cfg: QATConfig):
        self.cfg = cfg
        self.enabled = True
        self.calibrating = False
        self.input_amax: dict[str, torch.Tensor] = {}

    def applies(self, name: Optional[str]) -> bool:
        return self.enabled and name is not None and not any(fnmatchcase(name, p) for p in self.cfg.ignore)

    def weight(self, name: str, w: torch.Tensor) -> torch.Tensor:
        if self.cfg.weight is None:
            return w
        return w + (fake_quant(w.detach(), self.cfg.weight) - w).detach()

    def input(self, name: str, x: torch.Tensor) -> torch.Tensor:
        if self.calibrating:
            a = x.detach().abs().amax().float()
            prev = self.input_amax.get(name)
            self.input_amax[name] = a if prev is None else torch.maximum(prev, a)
            return x
        if self.cfg.input is None:
            return x
        amax = self.input_amax.get(name) if self.cfg.input.block is None or self.cfg.input.fmt == "nvfp4" else None
        return x + (fake_quant(x.detach(), self.cfg.input, amax) - x).detach()

    def quantizer_stats(self) -> dict:
        return {k: float(v) for k, v in sorted(self.input_amax.items())}


# ------------------------------------------------------------ NVFP4 storage
class NVFP4Tensor:
    """A weight in NVFP4 storage: e2m1 codes two per byte (low nibble = even
    column; bit 3 = sign, bits 0-2 = index into ``E2M1_VALUES``), one e4m3 scale
    per 16-element block of a row, one fp32 per-tensor scale."""

    def __init__(self, codes: torch.Tensor, block_scales: torch.Tensor, global_scale: float, shape: tuple):
        self.codes, self.block_scales, self.global_scale, self.shape = codes, block_scales, float(global_scale), shape

    @property
    def nbytes(self) -> int:
        return self.codes.numel() + self.block_scales.numel() + 4


def quant_nvfp4(w: torch.Tensor, amax: Optional[torch.Tensor] = None) -> NVFP4Tensor:
    """Real NVFP4 quantisation of a 2-D weight (rows x columns, columns padded to
    16): the same two-level scaling as the fake quantiser, so
    ``dequant_nvfp4(quant_nvfp4(w))`` equals ``fake_quant(w, nvfp4)``."""
    rows, cols = w.shape
    xf = w.float()
    a = amax if amax is not None else xf.abs().amax()
    g = float(a.clamp_min(1e-12)) / (6.0 * FP8_MAX)
    pc = -(-cols // 16) * 16
    if pc != cols:
        xf = torch.nn.functional.pad(xf, (0, pc - cols))
    b = xf.view(rows, pc // 16, 16)
    bs = _fp8_round(b.abs().amax(dim=2, keepdim=True) / 6.0 / g)   # e4m3 value of the block scale / g
    scale = (bs * g).clamp_min(1e-30)
    v = (b / scale).clamp(-6.0, 6.0)
    grid = E2M1_VALUES.to(w.device)
    idx = torch.bucketize(v.abs(), (grid[1:] + grid[:-1]) / 2)        # same rounding as _e2m1_round
    code = (idx | ((v < 0) & (idx > 0)).to(idx.dtype) << 3).to(torch.uint8).view(rows, pc)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    return NVFP4Tensor(packed.contiguous(), bs.view(rows, pc // 16).to(torch.float8_e4m3fn), g, (rows, cols))


def dequant_nvfp4(t: NVFP4Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    rows, cols = t.shape
    lo, hi = t.codes & 0x0F, t.codes >> 4
    code = torch.stack([lo, hi], -1).view(rows, -1).long()
    grid = E2M1_VALUES.to(t.codes.device)
    v = grid[code & 7] * torch.where(code >= 8, -1.0, 1.0)
    s = t.block_scales.float().repeat_interleave(16, 1) * t.global_scale
    return (v * s)[:, :cols].to(dtype)
