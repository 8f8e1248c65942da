"""Rank functions for the multi-process CPU (gloo) tests; importable by spawned ranks."""

import torch

from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.models.config import ModelConfig

TINY = ModelConfig(name="tiny-d", vocab_size=512, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                   head_dim=16, ffn_hidden_size=128, rope_theta=10000.0, max_position_embeddings=256)
TINY_MOE = ModelConfig(name="tiny-moe-d", vocab_size=512, hidden_size=64, num_layers=2, num_heads=4, num_kv_heads=2,
                       head_dim=16, ffn_hidden_size=0, rope_theta=10000.0, qk_norm=True, num_experts=8, moe_top_k=2,
                       moe_ffn_hidden_size=32, moe_aux_loss_coef=0.0, max_position_embeddings=256)


def make_batch(B=8, S=24, vocab=512, seed=0) -> BatchedDataDict:
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(S // 2, S + 1, (B,), generator=g)
    ids = torch.randint(0, vocab, (B, S), generator=g)
    tm = torch.zeros(B, S)
    for b in range(B):
        tm[b, 4:int(lens[b])] = 1
    adv = torch.randn(B, 1, generator=g).expand(B, S) * tm
    lp = -torch.rand(B, S, generator=g) * tm
    return BatchedDataDict({"input_ids": ids, "input_lengths": lens, "advantages": adv.contiguous(),
                            "generation_logprobs": lp, "prev_logprobs": lp.clone(), "token_mask": tm,
                            "sample_mask": torch.ones(B)})


def _pcfg(sp: bool):
    return {"max_total_sequence_length": 32, "precision": "float32", "train_global_batch_size": 8,
            "optimizer": {"kwargs": {"lr": 1e-3, "weight_decay": 0.01, "betas": [0.9, 0.999], "eps": 1e-8}},
            "megatron_cfg": {"sequence_parallel": sp},
            "generation": {"temperature": 1.0, "max_new_tokens": 4},
            "sequence_packing": {"train_mb_tokens": 64, "logprob_mb_tokens": 64}}


def case_train_step(rank: int, tp: int, ep: int, sp: bool, moe: bool):
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed

    torch.manual_seed(0)
    ps = init_distributed(tp=tp, ep=ep, backend="gloo")
    cfg = TINY_MOE if moe else TINY
    w = PolicyWorker(_pcfg(sp), model_cfg=cfg, pstate=ps, seed=3)
    full = make_batch()
    B = full.size
    per = B // ps.dp_size
    shard = full.slice(ps.dp_rank * per, (ps.dp_rank + 1) * per)
    res = w.train(shard, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=per)
    lp_after = w.get_logprobs(full)["logprobs"]
    return {"loss": res["loss"], "grad_norm": res["grad_norm"], "lp": lp_after,
            "probs_ratio_clamped_min": res.get("probs_ratio_clamped_min")}
