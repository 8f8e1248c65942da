"""Model architecture configs for the decoder families the framework trains and serves.

Shapes follow the public Hugging Face configs of the model families the
reference's recipes use (Llama-3.1-8B, Qwen3-30B-A3B, Qwen3-32B; reference
recipes ``examples/configs/grpo_math_8B*.yaml``,
``examples/configs/grpo_math_qwen30ba3b_megatron.yaml``), plus the tiny CPU model
of the plumbing run (2 layers, hidden 64, 4 heads / 2 KV heads, FFN 172,
vocab 512).  ``from_hf_config`` reads a HF ``config.json`` dict.
"""

from __future__ import annotations

import json
import os

import dataclasses
from dataclasses import dataclass, field
from typing import Optional

__all__ = ["ModelConfig", "PRESETS", "get_model_config"]


@dataclass
class ModelConfig:
    name: str = "custom"
    vocab_size: int = 512
    hidden_size: int = 64
    num_layers: int = 2
    num_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 16
    ffn_hidden_size: int = 172
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = None
    rms_eps: float = 1e-5
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    qk_norm: bool = False
    attention_bias: bool = False  # biases on the q / k / v projections (Qwen2)
    # Mixture of experts (0 experts = dense MLP)
    num_experts: int = 0
    moe_top_k: int = 0
    moe_ffn_hidden_size: int = 0
    moe_norm_topk_prob: bool = True
    moe_aux_loss_coef: float = 0.0
    moe_router_dtype: str = "fp32"
    # Draft head (speculative decoding): number of extra decoder layers of the
    # 1-layer draft head; 0 = none.
    draft_layers: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def num_params(self) -> int:
        H, V = self.hidden_size, self.vocab_size
        attn = H * (self.q_size + 2 * self.kv_size) + self.q_size * H
        if self.is_moe:
            mlp = self.num_experts * 3 * H * self.moe_ffn_hidden_size + self.num_experts * H
        else:
            mlp = 3 * H * self.ffn_hidden_size
        per_layer = attn + mlp + 2 * H + (2 * self.head_dim if self.qk_norm else 0)
        emb = V * H * (1 if self.tie_word_embeddings else 2)
        return self.num_layers * per_layer + emb + H

    def active_params_per_token(self) -> int:
        H = self.hidden_size
        attn = H * (self.q_size + 2 * self.kv_size) + self.q_size * H
        mlp = (self.moe_top_k * 3 * H * self.moe_ffn_hidden_size + self.num_experts * H) if self.is_moe \
            else 3 * H * self.ffn_hidden_size
        return self.num_layers * (attn + mlp) + self.vocab_size * H

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    @classmethod
    def from_hf_config(cls, hf: dict, name: str = "hf") -> "ModelConfig":
        H = hf["hidden_size"]
        nh = hf["num_attention_heads"]
        arch = (hf.get("architectures") or [""])[0].lower()
        n_exp = hf.get("num_experts", hf.get("num_local_experts", 0)) or 0
        return cls(
            name=name,
            vocab_size=hf["vocab_size"],
            hidden_size=H,
            num_layers=hf["num_hidden_layers"],
            num_heads=nh,
            num_kv_heads=hf.get("num_key_value_heads", nh),
            head_dim=hf.get("head_dim") or H // nh,
            ffn_hidden_size=hf.get("intermediate_size", 4 * H),
            rope_theta=float(hf.get("rope_theta", 10000.0)),
            rope_scaling=hf.get("rope_scaling"),
            rms_eps=float(hf.get("rms_norm_eps", 1e-5)),
            max_position_embeddings=hf.get("max_position_embeddings", 4096),
            tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
            qk_norm="qwen3" in arch or hf.get("model_type", "").startswith("qwen3"),
            attention_bias=bool(hf.get("attention_bias", hf.get("model_type", "") == "qwen2" or "qwen2" in arch)),
            num_experts=n_exp,
            moe_top_k=hf.get("num_experts_per_tok", 0) or 0,
            moe_ffn_hidden_size=hf.get("moe_intermediate_size", 0) or 0,
            moe_norm_topk_prob=bool(hf.get("norm_topk_prob", True)),
            moe_aux_loss_coef=float(hf.get("router_aux_loss_coef", 0.0) or 0.0),
        )

    def to_hf_config(self) -> dict:
        d = {
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.ffn_hidden_size,
            "rope_theta": self.rope_theta,
            "rope_scaling": self.rope_scaling,
            "rms_norm_eps": self.rms_eps,
            "max_position_embeddings": self.max_position_embeddings,
            "tie_word_embeddings": self.tie_word_embeddings,
            "torch_dtype": "bfloat16",
        }
        if self.attention_bias:
            d["attention_bias"] = True
        if self.is_moe:
            d.update({"architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
                      "num_experts": self.num_experts, "num_experts_per_tok": self.moe_top_k,
                      "moe_intermediate_size": self.moe_ffn_hidden_size, "norm_topk_prob": self.moe_norm_topk_prob,
                      "router_aux_loss_coef": self.moe_aux_loss_coef})
        elif self.qk_norm:
            d.update({"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3"})
        else:
            d.update({"architectures": ["LlamaForCausalLM"], "model_type": "llama"})
        return d


_LLAMA31_ROPE = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                 "original_max_position_embeddings": 8192}

PRESETS: dict[str, ModelConfig] = {
    "tiny-llama": ModelConfig(name="tiny-llama", vocab_size=512, hidden_size=64, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=16, ffn_hidden_size=172, rope_theta=10000.0,
                              max_position_embeddings=256),
    "tiny-moe": ModelConfig(name="tiny-moe", vocab_size=512, hidden_size=64, num_layers=2, num_heads=4,
                            num_kv_heads=2, head_dim=16, ffn_hidden_size=0, rope_theta=10000.0,
                            qk_norm=True, num_experts=8, moe_top_k=2, moe_ffn_hidden_size=48,
                            moe_aux_loss_coef=1e-3, max_position_embeddings=256),
    "qwen2.5-1.5b": ModelConfig(name="qwen2.5-1.5b", vocab_size=151936, hidden_size=1536, num_layers=28,
                                num_heads=12, num_kv_heads=2, head_dim=128, ffn_hidden_size=8960, rope_theta=1e6,
                                rms_eps=1e-6, max_position_embeddings=32768, tie_word_embeddings=True,
                                attention_bias=True),
    "qwen2.5-7b": ModelConfig(name="qwen2.5-7b", vocab_size=152064, hidden_size=3584, num_layers=28, num_heads=28,
                              num_kv_heads=4, head_dim=128, ffn_hidden_size=18944, rope_theta=1e6, rms_eps=1e-6,
                              max_position_embeddings=131072, attention_bias=True),
    "llama3.1-8b": ModelConfig(name="llama3.1-8b", vocab_size=128256, hidden_size=4096, num_layers=32,
                               num_heads=32, num_kv_heads=8, head_dim=128, ffn_hidden_size=14336,
                               rope_theta=500000.0, rope_scaling=dict(_LLAMA31_ROPE), rms_eps=1e-5,
                               max_position_embeddings=131072),
    "qwen3-30b-a3b": ModelConfig(name="qwen3-30b-a3b", vocab_size=151936, hidden_size=2048, num_layers=48,
                                 num_heads=32, num_kv_heads=4, head_dim=128, ffn_hidden_size=6144,
                                 rope_theta=1000000.0, rms_eps=1e-6, qk_norm=True, num_experts=128, moe_top_k=8,
                                 moe_ffn_hidden_size=768, moe_aux_loss_coef=1e-3, max_position_embeddings=40960),
    "qwen3-32b": ModelConfig(name="qwen3-32b", vocab_size=151936, hidden_size=5120, num_layers=64, num_heads=64,
                             num_kv_heads=8, head_dim=128, ffn_hidden_size=25600, rope_theta=1000000.0,
                             rms_eps=1e-6, qk_norm=True, max_position_embeddings=40960),
}


def get_model_config(name_or_cfg, **overrides) -> ModelConfig:
    if isinstance(name_or_cfg, ModelConfig):
        cfg = name_or_cfg
    elif isinstance(name_or_cfg, dict):
        cfg = ModelConfig(**name_or_cfg)
    elif os.path.isfile(os.path.join(str(name_or_cfg), "config.json")):
        # a Hugging Face model directory: the architecture from its config.json
        with open(os.path.join(str(name_or_cfg), "config.json")) as f:
            cfg = ModelConfig.from_hf_config(json.load(f), name=os.path.basename(str(name_or_cfg).rstrip("/")))
    else:
        key = str(name_or_cfg).lower()
        aliases = {
            "meta-llama/llama-3.1-8b-instruct": "llama3.1-8b",
            "meta-llama/llama-3.1-8b": "llama3.1-8b",
            "qwen/qwen3-30b-a3b": "qwen3-30b-a3b",
            "qwen/qwen2.5-1.5b": "qwen2.5-1.5b",
            "qwen/qwen2.5-7b": "qwen2.5-7b",
            "qwen/qwen3-32b": "qwen3-32b",
        }
        key = aliases.get(key, key)
        if key not in PRESETS:
            raise KeyError(f"unknown model preset {name_or_cfg!r}; known: {sorted(PRESETS)}")
        cfg = PRESETS[key]
    return cfg.replace(**overrides) if overrides else cfg


# HF config.json names that differ from the ModelConfig field names
_HF_NAMES = {"rms_norm_eps": "rms_eps", "num_hidden_layers": "num_layers", "num_attention_heads": "num_heads",
             "num_key_value_heads": "num_kv_heads", "intermediate_size": "ffn_hidden_size"}


def apply_hf_config_overrides(cfg: ModelConfig, overrides: Optional[dict], max_seq_len: Optional[int] = None
                              ) -> ModelConfig:
    """``policy.hf_config_overrides``: HF ``config.json`` keys that replace the
    model's settings for training and rollout alike (both run the same
    model).  ``rope_scaling`` with ``rope_type: yarn`` must give every YaRN
    field; it also sets ``rope_theta`` (when given) and widens
    ``max_position_embeddings`` to ``factor * original_max_position_embeddings``
    (and to ``max_seq_len``).

    Reference: ``policy.hf_config_overrides`` (``docs/guides/yarn-long-context.md``).
    """
    if not overrides:
        return cfg
    from rl_b200.ops.rope import YARN_FIELDS

    fields = {f for f in cfg.__dataclass_fields__}
    upd: dict = {}
    for k, v in overrides.items():
        name = _HF_NAMES.get(k, k)
        if name not in fields or name == "extra":
            raise ValueError(f"hf_config_overrides: unsupported key {k!r}")
        upd[name] = v
    rs = upd.get("rope_scaling")
    if rs is not None:
        rs = dict(rs)
        kind = rs.get("rope_type", rs.get("type"))
        if kind == "yarn":
            missing = [f for f in YARN_FIELDS if f not in rs or rs[f] is None]
            if missing:
                raise ValueError(f"hf_config_overrides.rope_scaling: YaRN needs every one of {list(YARN_FIELDS)}; "
                                 f"missing {missing}")
            if float(rs["factor"]) <= 0:
                raise ValueError("hf_config_overrides.rope_scaling.factor must be positive")
            upd["rope_theta"] = float(rs["rope_theta"])
            span = int(round(float(rs["factor"]) * int(rs["original_max_position_embeddings"])))
            upd["max_position_embeddings"] = max(int(upd.get("max_position_embeddings", cfg.max_position_embeddings)),
                                                 span)
        elif kind not in ("llama3", "default", None):
            raise ValueError(f"hf_config_overrides.rope_scaling: rope_type {kind!r} is not supported "
                             "(llama3, yarn)")
        upd["rope_scaling"] = rs
    if max_seq_len is not None:
        upd["max_position_embeddings"] = max(int(upd.get("max_position_embeddings", cfg.max_position_embeddings)),
                                             int(max_seq_len))
    return cfg.replace(**upd)

