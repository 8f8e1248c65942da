"""Router replay (R3): the rollout engine records the experts every MoE layer
picks for every processed token; training and log-prob forwards reuse them.

Reference behaviour: ``nemo_rl/models/megatron/router_replay.py`` (routes
recorded by the generation backend, replayed by the trainer's routers, missing
routes fall back to the computed top-k)."""

import os

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _moe_policy(**kw):
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY_MOE

    cfg = {"max_total_sequence_length": 48, "precision": "float32", "train_global_batch_size": 4,
           "optimizer": {"kwargs": {"lr": 1e-3, "weight_decay": 0.0}},
           "generation": {"temperature": 1.0, "max_new_tokens": 6, "mcore_generation_config": {"block_size_tokens": 8}},
           "sequence_packing": {"train_mb_tokens": 64, "logprob_mb_tokens": 64},
           "router_replay": {"enabled": True}}
    cfg.update(kw)
    return PolicyWorker(cfg, model_cfg=TINY_MOE, seed=4)


def test_engine_records_routes_and_training_replays_them():
    from tests.dist_cases import TINY_MOE

    w = _moe_policy()
    g = torch.Generator().manual_seed(0)
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (3, 10), generator=g),
                            "input_lengths": torch.tensor([10, 6, 8])})
    out = w.generate(data)
    R = out["routed_experts"]
    B, W = out["output_ids"].shape
    assert R.shape == (B, W, TINY_MOE.num_layers, TINY_MOE.moe_top_k)
    for b in range(B):
        n = int(out["unpadded_sequence_lengths"][b])
        assert (R[b, : n - 1] >= 0).all() and (R[b, : n - 1] < TINY_MOE.num_experts).all()
        assert (R[b, n - 1:] == -1).all()  # last sampled token and padding: no route

    # a forward over the rollout with the SAME weights picks the recorded experts
    seqs = BatchedDataDict({"input_ids": out["output_ids"], "input_lengths": out["unpadded_sequence_lengths"]})
    w.model.router_record = {}
    w._use_routes(BatchedDataDict())  # no replay
    w._forward_mb(seqs["input_ids"], [int(x) for x in seqs["input_lengths"]], [0], 1.0)
    rec = torch.stack([w.model.router_record[i] for i in range(TINY_MOE.num_layers)], 1).long()
    n0 = int(seqs["input_lengths"][0])
    assert torch.equal(torch.sort(rec[: n0 - 1], -1)[0], torch.sort(R[0, : n0 - 1].long(), -1)[0])

    # perturb the routers: without replay the choice changes, with replay it is the rollout's
    with torch.no_grad():
        for i in range(TINY_MOE.num_layers):
            gw = w.model.param(f"model.layers.{i}.mlp.gate.weight")
            gw.copy_(torch.randn(gw.shape, generator=g) * 3)
    w.model.router_record = {}
    w._forward_mb(seqs["input_ids"], [int(x) for x in seqs["input_lengths"]], [0], 1.0)
    free = torch.stack([w.model.router_record[i] for i in range(TINY_MOE.num_layers)], 1).long()
    assert not torch.equal(torch.sort(free[: n0 - 1], -1)[0], torch.sort(R[0, : n0 - 1].long(), -1)[0])
    seqs["routed_experts"] = R
    w._use_routes(seqs)
    w.model.router_record = {}
    w._forward_mb(seqs["input_ids"], [int(x) for x in seqs["input_lengths"]], [0], 1.0)
    rep = torch.stack([w.model.router_record[i] for i in range(TINY_MOE.num_layers)], 1).long()
    assert torch.equal(rep[: n0 - 1], R[0, : n0 - 1].long())
    # the token without a route fell back to the computed top-k
    assert torch.equal(rep[n0 - 1], free[n0 - 1])
    w._end_routes()
    w.model.router_record = None


def test_routes_flow_through_rollout_and_grpo_train_data():
    from rl_b200.algorithms.advantage_estimator import GRPOAdvantageEstimator
    from rl_b200.algorithms.grpo import build_train_data
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.environments.synthetic import HashRewardEnvironment
    from rl_b200.experience.rollouts import run_multi_turn_rollout

    w = _moe_policy()
    g = torch.Generator().manual_seed(1)
    logs = [[{"role": "user", "content": "", "token_ids": torch.randint(0, 512, (int(L),), generator=g)}]
            for L in (7, 9, 5, 8)]
    batch = BatchedDataDict({"message_log": logs, "task_name": ["synthetic"] * 4,
                             "extra_env_info": [None] * 4, "loss_multiplier": torch.ones(4)})
    rollout, _ = run_multi_turn_rollout(w, batch, None, {"synthetic": HashRewardEnvironment({})}, 48)
    for log in rollout["message_log"]:
        assert all("routed_experts" in m for m in log)
    data, _ = build_train_data(rollout, GRPOAdvantageEstimator({}, {}), {}, {}, torch.tensor([0, 0, 1, 1]))
    assert "routed_experts" in data and data["routed_experts"].shape[:2] == data["input_ids"].shape
    data["prev_logprobs"] = w.get_logprobs(data)["logprobs"]
    res = w.train(data, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=4)
    assert torch.isfinite(torch.tensor(res["loss"]))
    assert w._routes is None and w.model.router_replay is None
