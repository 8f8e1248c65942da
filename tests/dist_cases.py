"""Rank functions for the multi-process CPU (gloo) tests; importable by spawned ranks."""

from typing import Optional

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


def case_train_step(rank: int, tp: int, ep: int, sp: bool, moe: bool, cp: int = 1, pp: int = 1,
                    muon: Optional[dict] = None, mc_extra: Optional[dict] = None, num_layers: Optional[int] = None):
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed

    torch.manual_seed(0)
    ps = init_distributed(tp=tp, ep=ep, cp=cp, pp=pp, backend="gloo")
    cfg = TINY_MOE if moe else TINY
    if num_layers is not None:
        cfg = cfg.replace(num_layers=num_layers)
    pcfg = _pcfg(sp)
    if muon is not None:
        pcfg["megatron_cfg"]["optimizer"] = dict(muon)
    pcfg["megatron_cfg"].update(mc_extra or {})
    w = PolicyWorker(pcfg, model_cfg=cfg, pstate=ps, seed=3)
    full = make_batch()
    B = full.size
    per = B // ps.dp_size
    shard = full.slice(ps.dp_rank * per, (ps.dp_rank + 1) * per)
    res = w.train(shard, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=per)
    lp_after = w.get_logprobs(full)["logprobs"]
    return {"loss": res["loss"], "grad_norm": res["grad_norm"], "lp": lp_after,
            "probs_ratio_clamped_min": res.get("probs_ratio_clamped_min")}


def case_reshard_refit(rank: int, tp: int):
    """Training TP=tp, rollout TP=1: the resharded rollout copy equals the
    full-weight model of the same seed, before and after a training step, and
    the TP peers return the same rollouts."""
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.parallel.state import init_distributed, single_process_state

    torch.manual_seed(0)
    ps = init_distributed(tp=tp, backend="gloo")
    cfg = _pcfg(False)
    cfg["generation"] = dict(cfg["generation"], tensor_parallel_size=1)
    w = PolicyWorker(cfg, model_cfg=TINY, pstate=ps, seed=3)
    full = TransformerLM(TINY, single_process_state(), dtype=torch.float32, seed=3)
    init_err = (w.gen_model.flat_param - full.flat_param).abs().max().item()
    batch = make_batch()
    res = w.train(batch, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=batch.size)
    w.refit()
    # gather the trained shards and rebuild the full tensors independently
    errs = []
    for sp, p in w.model.named_flat_params():
        gp = w.gen_model.param(sp.name)
        if sp.tp_dim is None or tp == 1:
            errs.append((gp - p).abs().max().item())
            continue
        shards = [torch.empty_like(p) for _ in range(tp)]
        torch.distributed.all_gather(shards, p.detach().contiguous(), group=ps.tp_group)
        if sp.name.endswith(("qkv_proj.weight", "gate_up_proj.weight")):
            secs = 3 if "qkv" in sp.name else 2
            if secs == 3:
                hd, nq, nkv = TINY.head_dim, TINY.num_heads // tp, TINY.num_kv_heads // tp
                parts = [torch.split(s, [nq * hd, nkv * hd, nkv * hd], 0) for s in shards]
            else:
                parts = [s.chunk(2, 0) for s in shards]
            ref = torch.cat([torch.cat([pp[k] for pp in parts], 0) for k in range(secs)], 0)
        else:
            ref = torch.cat(shards, sp.tp_dim)
        errs.append((gp - ref).abs().max().item())
    data = BatchedDataDict({"input_ids": batch["input_ids"][:5, :8].clone(),
                            "input_lengths": torch.full((5,), 8, dtype=torch.long)})
    out = w.generate(data, greedy=True)
    return {"init_err": init_err, "refit_err": max(errs), "loss": res["loss"], "out_ids": out["output_ids"],
            "gen_lens": out["generation_lengths"]}


def case_pp_rollout_ckpt(rank: int, pp: int, tp: int, ckpt_dir: str):
    """Pipeline-parallel worker: the gathered full-depth rollout copy equals the
    training stages' weights after a step, greedy rollouts match the
    single-process worker's, and an HF checkpoint holds every stage's tensors."""
    from rl_b200.models.checkpoint_io import load_hf_checkpoint
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.parallel.state import init_distributed, single_process_state

    torch.manual_seed(0)
    ps = init_distributed(tp=tp, pp=pp, backend="gloo")
    w = PolicyWorker(_pcfg(False), model_cfg=TINY, pstate=ps, seed=3)
    batch = make_batch()
    w.train(batch, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=batch.size)
    w.refit()
    errs = [(w.gen_model.param(sp.name) - p).abs().max().item() for sp, p in w.model.named_flat_params()]
    data = BatchedDataDict({"input_ids": batch["input_ids"][:5, :8].clone(),
                            "input_lengths": torch.full((5,), 8, dtype=torch.long)})
    out = w.generate(data, greedy=True)
    w.save_checkpoint(ckpt_dir)
    w.save_checkpoint(ckpt_dir + "_dist", fmt="torch_dist")
    torch.distributed.barrier()
    full = TransformerLM(TINY, single_process_state(), dtype=torch.float32, seed=99)
    load_hf_checkpoint(full, ckpt_dir)
    ck_err = 0.0
    if tp == 1:
        # the HF checkpoint stores bf16
        ck_err = max((full.param(sp.name) - p.detach().to(torch.bfloat16).float()).abs().max().item()
                     for sp, p in w.model.named_flat_params())
    return {"sync_err": max(errs), "out_ids": out["output_ids"], "gen_lens": out["generation_lengths"],
            "ckpt_err": ck_err, "n_stage_params": len(w.model.specs), "n_gen_params": len(w.gen_model.specs),
            "gen_flat": w.gen_model.flat_param.detach().clone()}


def case_data_plane(rank: int, port: int):
    """Two processes share a Store-backed data plane: each consumes what the
    other produced."""
    from rl_b200.data_plane import StoreDataPlane

    dp = StoreDataPlane(host="127.0.0.1", port=port, is_master=rank == 0, world_size=2, compress=rank == 1)
    b = make_batch(B=4, S=12, seed=rank)
    b["names"] = [f"r{rank}-{i}" for i in range(4)]
    dp.put("train", f"from{rank}", b)
    got = dp.get("train", f"from{1 - rank}", timeout=60)
    ref = make_batch(B=4, S=12, seed=1 - rank)
    ok = all(torch.equal(got[k], ref[k]) for k in ref.keys()) and got["names"][0] == f"r{1 - rank}-0"
    keys = dp.keys("train")
    return {"ok": ok, "keys": keys, "stats": dp.metrics()}


def case_pp_exchange(rank: int, pp: int):
    """PipelineComm.exchange: a send to the next stage paired with a receive from
    it, and an unpaired send forward / receive from the previous stage."""
    from rl_b200.parallel.pipeline import PipelineComm
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(pp=pp, backend="gloo")
    comm = PipelineComm(ps)
    s = comm.stage
    cpu = torch.device("cpu")
    ok = True
    # unpaired: forward chain
    got = comm.exchange((torch.full((3,), float(s)), s + 1) if s + 1 < pp else None,
                        ((3,), torch.float32, cpu, s - 1) if s > 0 else None)
    ok &= got is None or float(got[0]) == s - 1
    comm.wait()
    # paired: even stages exchange with their next stage, odd ones with their previous
    peer = s + 1 if s % 2 == 0 else s - 1
    if 0 <= peer < pp:
        got = comm.exchange((torch.full((2,), 10.0 * s), peer), ((2,), torch.float32, cpu, peer))
        ok &= float(got[0]) == 10.0 * peer
    comm.wait()
    return {"rank": rank, "ok": bool(ok)}


def case_ckpt_relayout_vpp(rank: int, pp: int, path: str, vpp_save: int, vpp_load: int):
    """Save a sharded checkpoint under one virtual-pipeline setting and load it under
    another (same world / TP / PP sizes, different layers per rank)."""
    import torch.distributed as dist

    from rl_b200.models.checkpoint_io import load_dist_checkpoint, save_dist_checkpoint
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(pp=pp, backend="gloo")
    base = TINY.replace(num_layers=4)
    cfg_s = base.replace(extra={"virtual_pipeline_model_parallel_size": vpp_save})
    cfg_l = base.replace(extra={"virtual_pipeline_model_parallel_size": vpp_load})
    m_s = TransformerLM(cfg_s, ps, dtype=torch.float32, seed=5)
    save_dist_checkpoint(m_s, None, path, None)
    dist.barrier()
    m_l = TransformerLM(cfg_l, ps, dtype=torch.float32, seed=77)
    load_dist_checkpoint(m_l, None, path, None)
    saved = {sp.name: p.detach().clone() for sp, p in m_s.named_flat_params()}
    loaded = {sp.name: p.detach().clone() for sp, p in m_l.named_flat_params()}
    return {"saved": saved, "loaded": loaded}


def case_torch_dist(rank: int, tp: int, ep: int, moe: bool, path: str, mode: str):
    """torch_dist checkpoint round trip across layouts.  ``save``: one training step,
    save weights + optimizer, then a second step.  ``load``: a fresh worker (other
    seed) loads the checkpoint and takes the same second step.  Both return the
    HF-named weights at the checkpoint and the log-probs after the second step,
    so weights AND Adam moments must have moved across the layout change."""
    import torch.distributed as dist

    from rl_b200.models.checkpoint_io import hf_state_dict
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed

    torch.manual_seed(0)
    ps = init_distributed(tp=tp, ep=ep, backend="gloo")
    cfg = TINY_MOE if moe else TINY
    # MoE under TP runs with sequence parallelism, i.e. experts' FFN split over TP
    w = PolicyWorker(_pcfg(moe and tp > 1), model_cfg=cfg, pstate=ps, seed=3 if mode == "save" else 11)
    loss = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})

    def step(seed):
        full = make_batch(seed=seed)
        per = full.size // ps.dp_size
        w.train(full.slice(ps.dp_rank * per, (ps.dp_rank + 1) * per), loss, gbs=per)

    if mode == "save":
        step(0)
        w.save_checkpoint(path, optimizer_path=path + "_optimizer_flag", fmt="torch_dist")
    else:
        w.load_checkpoint(path, optimizer_path=path + "_optimizer_flag")
        # written again from the loading layout: must hold the same global tensors
        w.save_checkpoint(f"{path}_resaved_{tp}_{ep}_{ps.world_size}", optimizer_path="flag", fmt="torch_dist")
    sd = {k: v.detach().float().cpu().clone() for k, v in hf_state_dict(w.model, dtype=None).items()}
    step(1)
    lp = w.get_logprobs(make_batch(seed=2))["logprobs"]
    if dist.is_initialized():
        dist.barrier()
    return {"sd": sd, "lp": lp, "step": int(w.optimizer.step_count)}


def case_torch_dist_async(rank: int, tp: int, path: str):
    """Asynchronous torch_dist save: the weights are staged before save_checkpoint
    returns, so a training step taken right after does not leak into the files."""
    from rl_b200.models.checkpoint_io import hf_state_dict
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import init_distributed

    torch.manual_seed(0)
    ps = init_distributed(tp=tp, backend="gloo")
    w = PolicyWorker(_pcfg(False), model_cfg=TINY, pstate=ps, seed=3)
    loss = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    per = 8 // ps.dp_size
    w.train(make_batch(seed=0).slice(ps.dp_rank * per, (ps.dp_rank + 1) * per), loss, gbs=per)
    saved = {k: v.detach().float().cpu().clone() for k, v in hf_state_dict(w.model, dtype=None).items()}
    w.save_checkpoint(path, optimizer_path="flag", fmt="torch_dist", async_save=True)
    pending_after_return = not w.poll_async_save()
    w.train(make_batch(seed=1).slice(ps.dp_rank * per, (ps.dp_rank + 1) * per), loss, gbs=per)  # overlaps the write
    w.finalize_async_save()
    assert w.poll_async_save()
    w2 = PolicyWorker(_pcfg(False), model_cfg=TINY, pstate=ps, seed=9)
    w2.load_checkpoint(path, optimizer_path="flag")
    back = {k: v.detach().float().cpu().clone() for k, v in hf_state_dict(w2.model, dtype=None).items()}
    return {"max_err": max((back[k] - saved[k]).abs().max().item() for k in saved),
            "moved": max((back[k] - v.detach().float().cpu()).abs().max().item()
                         for k, v in hf_state_dict(w.model, dtype=None).items()),
            "pending": pending_after_return}


def case_single_controller_dp(rank: int):
    """Two gloo ranks; rank 1 drops a prompt: both train the same number of
    groups every step."""
    import torch.distributed as dist

    from rl_b200.algorithms.single_controller import RolloutDataError, SingleController
    from rl_b200.parallel.state import init_distributed
    from tests.test_single_controller_cpu import _fake_generate, _fake_train, _loader

    ps = init_distributed(backend="gloo")
    seen = []

    def fail(idx):
        if rank == 1 and 2 in idx:
            raise RolloutDataError("bad prompt on rank 1")

    sc = SingleController(_fake_generate([], fail), _fake_train(seen), _loader(12, per_batch=1), group_size=2,
                          groups_per_step=4, max_steps=2, dp_group=ps.dp_group,
                          cfg={"max_inflight_prompts": 1,
                               "rollout_failure": {"backoff_base_s": 0.0, "max_data_attempts_per_prompt": 1,
                                                   "max_skipped_prompts": 1, "min_step_batch_fraction": 0.75}})
    sc.run()
    dist.barrier()
    return [len(ix) for _, ix, _ in seen]
