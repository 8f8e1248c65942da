"""Logit parity with the HF implementations the checkpoints come from: tiny
random Llama / Qwen3 models built by ``transformers``, their state dicts
loaded into ``TransformerLM`` (``load_hf_state_dict``), compared in fp32 on
CPU, with default RoPE, Llama-3.1 frequency scaling and YaRN
(``policy.hf_config_overrides.rope_scaling``)."""

import pytest
import torch

transformers = pytest.importorskip("transformers")

from rl_b200.models.checkpoint_io import load_hf_state_dict
from rl_b200.models.config import ModelConfig, apply_hf_config_overrides
from rl_b200.models.transformer import TransformerLM
from rl_b200.ops.rope import rope_attention_factor, rope_inv_freq

YARN = {"rope_type": "yarn", "rope_theta": 10000.0, "factor": 4.0, "original_max_position_embeddings": 64,
        "truncate": True, "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 0.0}
LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 64}


def _hf_model(kind: str, rope_scaling):
    common = dict(vocab_size=256, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, max_position_embeddings=256, rms_norm_eps=1e-6,
                  rope_theta=10000.0, tie_word_embeddings=False, attention_bias=False)
    if rope_scaling is not None:
        common["rope_scaling"] = dict(rope_scaling)
    torch.manual_seed(0)
    if kind == "llama":
        cfg = transformers.LlamaConfig(**common)
        model = transformers.LlamaForCausalLM(cfg)
    elif kind == "qwen2":
        common.pop("attention_bias")
        common.pop("head_dim")
        cfg = transformers.Qwen2Config(**common)
        model = transformers.Qwen2ForCausalLM(cfg)
        with torch.no_grad():  # random (not zero) q / k / v biases
            for layer in model.model.layers:
                for proj in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj):
                    proj.bias.normal_(0, 0.5)
    else:
        cfg = transformers.Qwen3Config(**common)
        model = transformers.Qwen3ForCausalLM(cfg)
    return model.float().eval()


def _mine(kind: str, rope_scaling, sd, ps=None):
    cfg = ModelConfig(name="t", vocab_size=256, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=16, ffn_hidden_size=96, rope_theta=10000.0, rms_eps=1e-6, max_position_embeddings=256,
                      qk_norm=(kind == "qwen3"), attention_bias=(kind == "qwen2"))
    if rope_scaling is not None:
        cfg = apply_hf_config_overrides(cfg, {"rope_scaling": dict(rope_scaling)})
    m = TransformerLM(cfg, ps, device=torch.device("cpu"), dtype=torch.float32)
    load_hf_state_dict(m, sd)
    return m


@pytest.mark.parametrize("kind", ["llama", "qwen2", "qwen3"])
@pytest.mark.parametrize("scaling", [None, LLAMA3, YARN], ids=["default", "llama3", "yarn"])
def test_logits_match_hf(kind, scaling):
    if kind != "llama" and scaling is LLAMA3:
        pytest.skip("Llama-3.1 scaling belongs to Llama checkpoints")
    hf = _hf_model(kind, scaling)
    sd = {k: v.detach().clone() for k, v in hf.state_dict().items()}
    mine = _mine(kind, scaling, sd)
    g = torch.Generator().manual_seed(1)
    lens = [37, 150]  # the second sequence runs past the original 64-position context
    ids = [torch.randint(0, 256, (L,), generator=g) for L in lens]
    with torch.no_grad():
        ref = [hf(x.view(1, -1)).logits[0] for x in ids]
        flat = torch.cat(ids)
        pos = torch.cat([torch.arange(L) for L in lens])
        cu = torch.tensor([0, lens[0], sum(lens)], dtype=torch.int32)
        h = mine(flat, pos, cu, max(lens))
        got = mine.logits(h)
    ref = torch.cat(ref)
    err = (got - ref).abs().max().item()
    assert err < 2e-4 * max(1.0, ref.abs().max().item()), err


def test_yarn_matches_transformers_frequencies():
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    for sc, hd in [({**YARN, "rope_theta": 1e6, "factor": 3.2, "original_max_position_embeddings": 40960}, 128),
                   ({**YARN, "rope_theta": 1e4, "factor": 8.0, "original_max_position_embeddings": 4096,
                     "truncate": False, "mscale": 0.707, "mscale_all_dim": 0.707}, 128),
                   ({**YARN, "rope_theta": 5e5, "beta_fast": 16.0, "beta_slow": 2.0, "mscale_all_dim": 1.0}, 64)]:
        c = transformers.Qwen2Config(hidden_size=hd * 4, num_attention_heads=4, rope_scaling=dict(sc),
                                     max_position_embeddings=int(sc["factor"] * sc["original_max_position_embeddings"]))
        inv, att = ROPE_INIT_FUNCTIONS["yarn"](c)
        mine = rope_inv_freq(hd, sc["rope_theta"], sc)
        assert torch.allclose(mine.double(), inv.double(), rtol=1e-6, atol=0)
        assert abs(rope_attention_factor(sc) - att) < 1e-12


def test_hf_config_overrides_validation():
    base = ModelConfig()
    with pytest.raises(ValueError, match="missing"):
        apply_hf_config_overrides(base, {"rope_scaling": {"rope_type": "yarn", "factor": 2.0}})
    with pytest.raises(ValueError, match="unsupported key"):
        apply_hf_config_overrides(base, {"not_a_field": 1})
    with pytest.raises(ValueError, match="not supported"):
        apply_hf_config_overrides(base, {"rope_scaling": {"rope_type": "dynamic", "factor": 2.0}})
    cfg = apply_hf_config_overrides(base, {"rope_scaling": dict(YARN, original_max_position_embeddings=4096)},
                                    max_seq_len=8192)
    assert cfg.max_position_embeddings == 16384 and cfg.rope_theta == 10000.0
    cfg = apply_hf_config_overrides(base, {"rms_norm_eps": 1e-6})
    assert cfg.rms_eps == 1e-6


def test_worker_applies_overrides():
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY, _pcfg

    cfg = _pcfg(False)
    cfg["max_total_sequence_length"] = 512
    with pytest.raises(ValueError, match="rotary positions"):
        PolicyWorker(cfg, model_cfg=TINY, seed=3)  # TINY has 256 positions
    cfg["hf_config_overrides"] = {"rope_scaling": dict(YARN, original_max_position_embeddings=128)}
    w = PolicyWorker(cfg, model_cfg=TINY, seed=3)
    assert w.model.rope_cache.shape[0] >= 512 and w.model_cfg.rope_scaling["rope_type"] == "yarn"
    assert w.gen_model.rope_cache is w.model.rope_cache or torch.equal(w.gen_model.rope_cache, w.model.rope_cache)


def _tp2_qwen2(rank):
    """Qwen2 (q / k / v biases) at TP=2: logits gathered over the vocab shards
    equal HF's, and the HF state dict round-trips through the TP shards."""
    import torch.distributed as dist

    from rl_b200.models.checkpoint_io import hf_state_dict
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(tp=2, backend="gloo")
    hf = _hf_model("qwen2", None)
    sd = {k: v.detach().clone() for k, v in hf.state_dict().items()}
    mine = _mine("qwen2", None, sd, ps)
    ids = torch.randint(0, 256, (40,), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        ref = hf(ids.view(1, -1)).logits[0]
        h = mine(ids, torch.arange(40), torch.tensor([0, 40], dtype=torch.int32), 40)
        loc = mine.logits(h)
        parts = [torch.empty_like(loc) for _ in range(2)]
        dist.all_gather(parts, loc.contiguous(), group=ps.tp_group)
    back = hf_state_dict(mine, dtype=None)
    same = all(torch.equal(back[k], sd[k]) for k in sd if k in back)
    return {"err": float((torch.cat(parts, -1) - ref).abs().max()), "roundtrip": same,
            "bias_keys": sorted(k for k in back if k.endswith("q_proj.bias"))}


def test_qwen2_tp2_matches_hf():
    from rl_b200.distributed.launch import spawn_ranks

    outs = spawn_ranks(_tp2_qwen2, 2)
    for o in outs:
        assert o["err"] < 2e-4 and o["roundtrip"] and len(o["bias_keys"]) == 2, o
