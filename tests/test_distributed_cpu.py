"""Tensor / sequence / data / expert parallelism on CPU gloo ranks, each compared with
a single-process run of the same step (same seed, same global batch).

Mirrors the reference's distributed unit-test strategy (spawned localhost ranks
compared against a single-device baseline, ``tests/unit/distributed/test_distributed_logprob.py``)."""

import pytest
import torch

from rl_b200.distributed.launch import spawn_ranks
from tests.dist_cases import case_train_step


@pytest.fixture(scope="module")
def dense_single():
    return spawn_ranks(case_train_step, 1, 1, 1, False, False)[0]


@pytest.fixture(scope="module")
def moe_single():
    return spawn_ranks(case_train_step, 1, 1, 1, False, True)[0]


def _close(a, b, tol=2e-4):
    assert abs(a["loss"] - b["loss"]) < tol * max(1.0, abs(b["loss"])), (a["loss"], b["loss"])
    assert abs(a["grad_norm"] - b["grad_norm"]) < tol * max(1.0, b["grad_norm"]), (a["grad_norm"], b["grad_norm"])
    assert torch.allclose(a["lp"], b["lp"], atol=5e-4), (a["lp"] - b["lp"]).abs().max()


@pytest.mark.parametrize("world,tp,sp", [(2, 2, False), (2, 2, True), (2, 1, False), (4, 2, False), (4, 2, True)])
def test_dense_parallel_matches_single(dense_single, world, tp, sp):
    outs = spawn_ranks(case_train_step, world, tp, 1, sp, False)
    for o in outs:
        _close(o, dense_single)


@pytest.mark.parametrize("world,tp,ep,sp,extra", [
    (2, 2, 1, True, None),                                   # SP: experts' FFN split over TP (ETP = TP)
    (2, 2, 1, False, {"expert_tensor_parallel_size": 2}),   # ETP without SP
    (2, 2, 1, False, None),                                  # whole experts replicated over TP
    (4, 2, 2, True, None),                                   # ETP x EP
])
def test_moe_expert_tensor_parallel_matches_single(moe_single, world, tp, ep, sp, extra):
    outs = spawn_ranks(case_train_step, world, tp, ep, sp, True, 1, 1, None, extra)
    for o in outs:
        _close(o, moe_single)


def test_moe_expert_parallel_matches_single(moe_single):
    outs = spawn_ranks(case_train_step, 2, 1, 2, False, True)
    for o in outs:
        _close(o, moe_single)


def test_reshard_refit_tp2_to_rollout_tp1():
    from tests.dist_cases import case_reshard_refit

    outs = spawn_ranks(case_reshard_refit, 2, 2)
    for o in outs:
        assert o["init_err"] == 0.0, o["init_err"]
        assert o["refit_err"] == 0.0, o["refit_err"]
    assert torch.equal(outs[0]["out_ids"], outs[1]["out_ids"])
    assert outs[0]["out_ids"].shape[0] == 5


@pytest.mark.parametrize("world,tp,cp,sp", [(2, 1, 2, False), (4, 2, 2, True), (4, 1, 2, False)])
def test_context_parallel_matches_single(dense_single, world, tp, cp, sp):
    """Load-balanced CP chunks + gathered-KV attention reproduce the single-process step."""
    outs = spawn_ranks(case_train_step, world, tp, 1, sp, False, cp)
    for o in outs:
        _close(o, dense_single)


@pytest.mark.parametrize("world,tp,pp", [(2, 1, 2), (4, 2, 2), (4, 1, 2)])
def test_pipeline_parallel_matches_single(dense_single, world, tp, pp):
    """1F1B pipeline over 2 stages (with TP or DP beside it): loss, grad norm
    and log-probs after the step match the single-process run."""
    outs = spawn_ranks(case_train_step, world, tp, 1, False, False, 1, pp)
    for o in outs:
        _close(o, dense_single)


def test_pipeline_rollout_refit_and_checkpoint(tmp_path):
    from tests.dist_cases import case_pp_rollout_ckpt

    outs = spawn_ranks(case_pp_rollout_ckpt, 2, 2, 1, str(tmp_path / "hf"))
    for o in outs:
        assert o["sync_err"] == 0.0
        assert o["ckpt_err"] < 1e-6
        assert o["n_stage_params"] < o["n_gen_params"]
    torch.testing.assert_close(outs[0]["gen_flat"], outs[1]["gen_flat"], atol=0, rtol=0)
    assert torch.equal(outs[0]["out_ids"], outs[1]["out_ids"])
    # the sharded checkpoint of the 2 stages re-lays out into one full model
    from rl_b200.models.checkpoint_io import load_dist_checkpoint
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.parallel.state import single_process_state
    from tests.dist_cases import TINY

    full = TransformerLM(TINY, single_process_state(), dtype=torch.float32, seed=99)
    load_dist_checkpoint(full, None, str(tmp_path / "hf_dist"), None)
    n = outs[0]["gen_flat"].numel()
    torch.testing.assert_close(full.flat_param[:n], outs[0]["gen_flat"], atol=0, rtol=0)


def test_schedule_1f1b_order():
    from rl_b200.parallel.pipeline import schedule_1f1b

    for S in (2, 3, 4):
        for M in (1, 2, 5, 8):
            for s in range(S):
                acts = schedule_1f1b(S, s, M)
                assert [i for k, i in acts if k == "F"] == list(range(M))
                assert [i for k, i in acts if k == "B"] == list(range(M))
                live = peak = 0
                for k, i in acts:
                    live += 1 if k == "F" else -1
                    peak = max(peak, live)
                    assert k == "F" or ("F", i) in acts[:acts.index((k, i))]
                assert peak <= min(S - s, M)


def test_pipeline_plans_cannot_deadlock_under_rendezvous():
    """The plans finish when every send of a large message waits for its
    receive (NCCL past its channel buffer), each rank pair's communicator runs
    its point-to-point work in posting order, and the executor pairs a step's
    send with the next step's receive to the same peer in one group.  Posting
    them separately deadlocks 1F1B at two stages and the interleaved schedule."""
    from rl_b200.parallel.pipeline import plan_1f1b, plan_virtual, simulate_rendezvous

    for S in (2, 3, 4):
        for M in (1, 2, 3, 4, 5, 8, 13):
            assert simulate_rendezvous([plan_1f1b(S, s, M) for s in range(S)]), (S, M)
            assert simulate_rendezvous([plan_1f1b(S, s, M, backward=False) for s in range(S)]), (S, M)
            for V in (2, 3):
                for bw in (True, False):
                    assert simulate_rendezvous([plan_virtual(S, s, M, V, bw) for s in range(S)]), (S, M, V, bw)
    # the hazard the pairing removes
    assert not simulate_rendezvous([plan_1f1b(2, s, 4) for s in range(2)], pair_same_peer=False)
    assert not simulate_rendezvous([plan_virtual(2, s, 4, 2) for s in range(2)], pair_same_peer=False)


def test_pipeline_comm_exchange():
    """Sends and receives between stages over gloo, paired and unpaired."""
    from tests.dist_cases import case_pp_exchange

    outs = spawn_ranks(case_pp_exchange, 3, 3)
    for o in outs:
        assert o["ok"], o


def test_uneven_pipeline_stages():
    """``num_layers_in_first/last_pipeline_stage``: 5 layers as 1 | 2 | 2 and
    3 | 2 over 3 / 2 stages train like the single-process model."""
    from rl_b200.models.transformer import stage_layers

    assert [list(stage_layers(5, 3, r, first=1)) for r in range(3)] == [[0], [1, 2], [3, 4]]
    assert [list(stage_layers(5, 2, r, first=3)) for r in range(2)] == [[0, 1, 2], [3, 4]]
    assert [list(stage_layers(8, 3, r, first=2, last=2)) for r in range(3)] == [[0, 1], [2, 3, 4, 5], [6, 7]]
    with pytest.raises(ValueError):
        stage_layers(6, 3, 0, first=1)  # 5 layers left for 2 stages
    single = spawn_ranks(case_train_step, 1, 1, 1, False, False, 1, 1, None, None, 5)[0]
    for world, extra in [(3, {"num_layers_in_first_pipeline_stage": 1}),
                         (2, {"num_layers_in_first_pipeline_stage": 3})]:
        outs = spawn_ranks(case_train_step, world, 1, 1, False, False, 1, world, None, extra, 5)
        for o in outs:
            _close(o, single)


@pytest.mark.parametrize("world,layers", [(2, 4), (3, 6)])
def test_virtual_pipeline_matches_single(world, layers):
    """``virtual_pipeline_model_parallel_size: 2``: each rank holds two
    interleaved layer chunks (rank r: chunks r and r + pp); training step and
    log-probs equal the single-process run."""
    single = spawn_ranks(case_train_step, 1, 1, 1, False, False, 1, 1, None, None, layers)[0]
    outs = spawn_ranks(case_train_step, world, 1, 1, False, False, 1, world, None,
                       {"virtual_pipeline_model_parallel_size": 2}, layers)
    for o in outs:
        _close(o, single)


def test_dist_checkpoint_across_virtual_pipeline_settings(tmp_path):
    """A checkpoint saved with two layer chunks per rank (rank 0 holds layers 0
    and 2) loads under one chunk per rank (rank 0 holds layers 0 and 1): every
    parameter arrives under its own name, not by flat-buffer position."""
    from tests.dist_cases import case_ckpt_relayout_vpp

    for vs, vl in ((2, 1), (1, 2)):
        d = tmp_path / f"v{vs}{vl}"
        outs = spawn_ranks(case_ckpt_relayout_vpp, 2, 2, str(d), vs, vl)
        saved = {k: v for o in outs for k, v in o["saved"].items()}
        loaded = {k: v for o in outs for k, v in o["loaded"].items()}
        assert saved.keys() == loaded.keys()
        for k in saved:
            torch.testing.assert_close(loaded[k], saved[k], atol=0, rtol=0, msg=k)


@pytest.mark.parametrize("moe,save,loads", [
    (False, (2, 2, 1), [(1, 1, 1), (2, 1, 1), (4, 2, 1)]),   # (world, tp, ep): TP=2 -> 1 GPU, DP=2, TP2 x DP2
    (True, (2, 1, 2), [(1, 1, 1), (2, 2, 1)]),               # EP=2 -> 1 GPU, TP=2
    (True, (4, 2, 2), [(1, 1, 1), (2, 1, 2)]),               # TP2 x EP2 with split experts -> 1 GPU, EP2
])
def test_torch_dist_checkpoint_relayout(tmp_path, moe, save, loads):
    """A Megatron torch_dist checkpoint (DCP shards under Megatron names, optimizer
    embedded) saved at one layout resumes at others: the same weights, a
    checkpoint written again from the new layout holds bit-identical global
    tensors (weights, fp32 master, both Adam moments), and the next training
    step gives the same log-probs as continuing at the saving layout (MoE:
    within the tolerance of the TP / EP step itself, whose near-zero expert
    gradients Adam normalises)."""
    import torch.distributed.checkpoint as dcp

    from rl_b200.models.megatron_ckpt import read_global_tensor
    from tests.dist_cases import case_torch_dist

    path = str(tmp_path / "weights")
    ref = spawn_ranks(case_torch_dist, save[0], save[1], save[2], moe, path, "save")[0]
    it = tmp_path / "weights" / "iter_0000000"
    assert (it / "metadata.json").exists() and (it / "common.pt").exists() and (it / ".metadata").exists()
    assert list(it.glob("__*_*.distcp"))
    for world, tp, ep in loads:
        outs = spawn_ranks(case_torch_dist, world, tp, ep, moe, path, "load")
        for o in outs:
            assert o["sd"].keys() == ref["sd"].keys()
            for k in ref["sd"]:
                torch.testing.assert_close(o["sd"][k], ref["sd"][k], atol=0, rtol=0, msg=k)
            assert o["step"] == ref["step"]
            tol = 5e-3 if moe else 5e-4
            assert torch.allclose(o["lp"], ref["lp"], atol=tol), (world, tp, ep, (o["lp"] - ref["lp"]).abs().max())
        again = f"{path}_resaved_{tp}_{ep}_{world}"
        keys = dcp.FileSystemReader(f"{path}/iter_0000000").read_metadata().state_dict_metadata.keys()
        assert any(k.startswith("optimizer.state.exp_avg_sq.") for k in keys)
        for k in keys:
            torch.testing.assert_close(read_global_tensor(again, k), read_global_tensor(path, k), atol=0, rtol=0,
                                       msg=k)


def test_torch_dist_megatron_layout(tmp_path):
    """The stacked Megatron tensors: QKV rows grouped per KV head ([q heads of the
    group, k, v]), fc1 = [gate; up], layer index leading."""
    from rl_b200.models.megatron_ckpt import read_global_tensor
    from tests.dist_cases import TINY, case_torch_dist

    path = str(tmp_path / "w")
    ref = spawn_ranks(case_torch_dist, 2, 2, 1, False, path, "save")[0]["sd"]
    c = TINY
    qpg, hd, H = c.num_heads // c.num_kv_heads, c.head_dim, c.hidden_size
    qkv = read_global_tensor(path, "decoder.layers.self_attention.linear_qkv.weight")
    assert qkv.shape == (c.num_layers, (c.num_heads + 2 * c.num_kv_heads) * hd, H)
    for layer in range(c.num_layers):
        g = qkv[layer].float().view(c.num_kv_heads, qpg + 2, hd, H)
        pre = f"model.layers.{layer}.self_attn."
        torch.testing.assert_close(g[:, :qpg], ref[pre + "q_proj.weight"].view(c.num_kv_heads, qpg, hd, H))
        torch.testing.assert_close(g[:, qpg], ref[pre + "k_proj.weight"].view(c.num_kv_heads, hd, H))
        torch.testing.assert_close(g[:, qpg + 1], ref[pre + "v_proj.weight"].view(c.num_kv_heads, hd, H))
    fc1 = read_global_tensor(path, "decoder.layers.mlp.linear_fc1.weight")
    torch.testing.assert_close(fc1[1].float(), torch.cat([ref["model.layers.1.mlp.gate_proj.weight"],
                                                          ref["model.layers.1.mlp.up_proj.weight"]]))
    emb = read_global_tensor(path, "embedding.word_embeddings.weight")
    torch.testing.assert_close(emb.float(), ref["model.embed_tokens.weight"])
    exp_avg = read_global_tensor(path, "optimizer.state.exp_avg.decoder.layers.self_attention.linear_proj.weight")
    assert exp_avg.shape == (c.num_layers, H, c.num_heads * hd) and exp_avg.abs().sum() > 0


@pytest.mark.parametrize("world,tp", [(1, 1), (2, 2)])
def test_torch_dist_async_save(tmp_path, world, tp):
    """Background torch_dist writes (gloo coordination group, host-staged pieces):
    the files hold the weights of the moment of the call even though training
    continues during the write."""
    from tests.dist_cases import case_torch_dist_async

    outs = spawn_ranks(case_torch_dist_async, world, tp, str(tmp_path / "w"))
    for o in outs:
        assert o["max_err"] == 0.0 and o["moved"] > 0.0
