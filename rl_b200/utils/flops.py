"""Model FLOPs accounting and MFU.

Reference: ``FLOPTracker`` / ``THEORETICAL_TFLOPS`` (``nemo_rl/utils/flops_tracker.py``,
table ``:210``) with per-family formulas (``nemo_rl/utils/flops_formulas.py``: llama
``:77``, qwen3 ``:174``) and the per-stage throughput / MFU report of
``print_performance_metrics`` (``nemo_rl/algorithms/utils.py:605``).

Forward FLOPs of one packed sequence of length ``s`` for the decoder family
implemented here (dense SwiGLU or top-k MoE, GQA, untied or tied LM head):

    per layer: 2 s H (q + 2 kv + o projections)           -> 2 s H (H + 2 nkv hd + H)   [nq hd = H]
               2 s * 3 H F (gate, up, down)                (dense)
               2 s * k * 3 H F_e + 2 s H E                  (MoE: top-k experts + router)
               2 * 2 * s^2/2 * nq hd                        (causal QK^T and PV)
    head:      2 s H V

Training = forward + backward (2x forward) = 3x forward (+1x with activation
recomputation).  Peaks are dense (no 2:4 sparsity) per GPU, TFLOP/s.
"""

from __future__ import annotations

from typing import Iterable, Optional

__all__ = ["THEORETICAL_TFLOPS", "forward_flops", "FLOPTracker", "mfu"]

THEORETICAL_TFLOPS = {
    ("B200", "bf16"): 2250.0, ("B200", "fp8"): 4500.0, ("B200", "fp4"): 9000.0,
    ("GB200", "bf16"): 2500.0, ("GB200", "fp8"): 5000.0,
    ("H100", "bf16"): 989.0, ("H100", "fp8"): 1979.0,
    ("H200", "bf16"): 989.0, ("H200", "fp8"): 1979.0,
    ("A100", "bf16"): 312.0,
}


def forward_flops(cfg, seq_lens: Iterable[int]) -> float:
    H, L, V = cfg.hidden_size, cfg.num_layers, cfg.vocab_size
    hd, nq, nkv = cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    attn_proj = 2 * H * (nq * hd + 2 * nkv * hd) + 2 * nq * hd * H
    if cfg.num_experts:
        mlp = 2 * cfg.moe_top_k * 3 * H * cfg.moe_ffn_hidden_size + 2 * H * cfg.num_experts
    else:
        mlp = 2 * 3 * H * cfg.ffn_hidden_size
    per_tok = L * (attn_proj + mlp) + 2 * H * V
    tot = 0.0
    for s in seq_lens:
        s = float(s)
        tot += s * per_tok + L * 2.0 * s * s * nq * hd  # causal: 2 GEMMs x s^2/2 x nq x hd x 2
    return tot


def device_name() -> str:
    try:
        import torch

        if torch.cuda.is_available():
            n = torch.cuda.get_device_name()
            for k in ("GB200", "B200", "H200", "H100", "A100"):
                if k in n:
                    return k
    except Exception:  # noqa: BLE001
        pass
    return "B200"


def mfu(flops: float, seconds: float, n_gpus: int, dtype: str = "bf16", device: Optional[str] = None) -> float:
    peak = THEORETICAL_TFLOPS.get((device or device_name(), dtype), THEORETICAL_TFLOPS[("B200", "bf16")])
    return flops / max(seconds, 1e-12) / max(1, n_gpus) / (peak * 1e12)


class FLOPTracker:
    """Accumulates model FLOPs of the sequences a stage processed."""

    def __init__(self, cfg, recompute: bool = False):
        self.cfg = cfg
        self.recompute = recompute
        self.fwd = 0.0

    def reset(self) -> None:
        self.fwd = 0.0

    def track(self, seq_lens: Iterable[int]) -> float:
        f = forward_flops(self.cfg, seq_lens)
        self.fwd += f
        return f

    def train_flops(self) -> float:
        return self.fwd * (4.0 if self.recompute else 3.0)

    def model_train_flops(self) -> float:
        """Without recomputation (the convention for MFU)."""
        return self.fwd * 3.0
