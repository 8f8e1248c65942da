"""LoRA adapters: start equal to the base, train only the adapters, merge into
the rollout copy, reference policy = base, PEFT round trip, and TP=2 (gloo)
matching a single process."""

import torch

from rl_b200.distributed.launch import spawn_ranks
from tests.dist_cases import TINY, make_batch


def _pcfg(lora=True, **kw):
    c = {"max_total_sequence_length": 32, "precision": "float32", "train_global_batch_size": 8,
         "optimizer": {"kwargs": {"lr": 5e-3, "weight_decay": 0.0}},
         "generation": {"temperature": 1.0, "max_new_tokens": 4},
         "sequence_packing": {"train_mb_tokens": 64, "logprob_mb_tokens": 64},
         "lora_cfg": {"enabled": lora, "dim": 4, "alpha": 8}}
    c.update(kw)
    return c


def test_lora_train_merge_reference_and_peft(tmp_path):
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.policy.worker import PolicyWorker

    data = make_batch(B=8, S=24, seed=2)
    base = PolicyWorker(_pcfg(lora=False), model_cfg=TINY, seed=5)
    w = PolicyWorker(_pcfg(), model_cfg=TINY, seed=5)
    lp0 = base.get_logprobs(data)["logprobs"]
    assert torch.allclose(w.get_logprobs(data)["logprobs"], lp0, atol=1e-6)  # B = 0 at init
    flat_before = w.model.flat_param.clone()
    lf = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    for _ in range(3):
        w.train(data, lf, gbs=8)
    assert torch.equal(w.model.flat_param, flat_before)  # base frozen
    assert w.lora.flat_param.abs().sum() > 0
    lp1 = w.get_logprobs(data)["logprobs"]
    assert (lp1 - lp0).abs().max() > 1e-4
    # reference policy = base
    ref = w.get_reference_policy_logprobs(data)["reference_logprobs"]
    assert torch.allclose(ref, lp0, atol=1e-6)
    # the rollout copy holds the merged weights: its logits equal the adapted model's
    w.refit()
    name = "model.layers.0.self_attn.qkv_proj.weight"
    an, bn = w.lora.layers[name]
    merged = w.model.param(name) + w.lora.scale * (w.lora._params[bn] @ w.lora._params[an])
    assert torch.allclose(w.gen_model.param(name), merged, atol=1e-6)
    # PEFT round trip
    w.save_checkpoint(str(tmp_path / "adapter"))
    w2 = PolicyWorker(_pcfg(), model_cfg=TINY, seed=5)
    w2.load_checkpoint(str(tmp_path / "adapter"))
    assert torch.allclose(w2.get_logprobs(data)["logprobs"], lp1, atol=1e-5)
    assert (tmp_path / "adapter" / "adapter_config.json").exists()


def _case_lora_tp(rank: int, tp: int):
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(tp=tp, backend="gloo")
    w = PolicyWorker(_pcfg(), model_cfg=TINY, pstate=ps, seed=5)
    data = make_batch(B=8, S=24, seed=2)
    res = [w.train(data, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=8) for _ in range(2)]
    return {"loss": [r["loss"] for r in res], "gn": [r["grad_norm"] for r in res],
            "lp": w.get_logprobs(data)["logprobs"]}


def test_lora_tp2_matches_single():
    one = spawn_ranks(_case_lora_tp, 1, 1)[0]
    two = spawn_ranks(_case_lora_tp, 2, 2)
    for o in two:
        for a, b in zip(o["loss"], one["loss"]):
            assert abs(a - b) < 2e-4 * max(1, abs(b))
        for a, b in zip(o["gn"], one["gn"]):
            assert abs(a - b) < 2e-4 * max(1, b), (o["gn"], one["gn"])
        assert torch.allclose(o["lp"], one["lp"], atol=5e-4)
