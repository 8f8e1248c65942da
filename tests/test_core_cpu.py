"""CPU unit tests of the framework layer (no GPU): configs, batch containers, packing,
losses, advantage estimators, checkpoint formats, environments and training loops."""

import json
import math
import os
import random

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# ------------------------------------------------------------------ config
def test_config_inheritance_interpolation_overrides(tmp_path):
    from rl_b200.utils.config import load_config

    cfg = load_config(os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
                      ["grpo.seed=7", "+policy.new_key=3", "~logger.monitor_gpus"])
    assert cfg["grpo"]["seed"] == 7
    assert cfg["policy"]["new_key"] == 3
    assert "monitor_gpus" not in cfg["logger"]
    # ${mul:...} resolver and ${a.b} interpolation
    assert cfg["policy"]["sequence_packing"]["train_mb_tokens"] == 32 * 4
    assert cfg["grpo"]["reward_shaping"]["max_response_length"] == 32
    assert cfg["grpo"]["adv_estimator"]["normalize_rewards"] is True
    with pytest.raises(KeyError):
        load_config(os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"), ["grpo.not_a_key=1"])
    for f in os.listdir(os.path.join(ROOT, "examples", "configs")):
        load_config(os.path.join(ROOT, "examples", "configs", f))


# ------------------------------------------------------- BatchedDataDict
def test_batched_data_dict_shard_and_microbatch():
    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    B, S = 16, 10
    d = BatchedDataDict({"x": torch.arange(B * S).view(B, S), "lens": torch.tensor([2 + i % 8 for i in range(B)]),
                         "tags": [f"t{i}" for i in range(B)]})
    shards = d.shard_by_batch_size(4, batch_size=8)
    assert [s.size for s in shards] == [4, 4, 4, 4]
    # shard 0 holds rows 0,1 of each global batch of 8
    assert shards[0]["tags"] == ["t0", "t1", "t8", "t9"]
    back = BatchedDataDict.from_batches(shards)
    assert back.size == B
    mbs = list(d.make_microbatch_iterator(5))
    assert [m.size for m in mbs] == [5, 5, 5, 1]
    sh, order = d.shard_by_batch_size(2, batch_size=16, dynamic_batching_args={
        "max_tokens_per_microbatch": 16, "sequence_length_round": 4, "input_lengths_key": "lens", "input_key": "x"})
    for s in sh:
        for mb in s.make_microbatch_iterator_with_dynamic_shapes():
            assert mb["x"].shape[1] * mb.size <= 16 or mb.size == 1
    back = BatchedDataDict.from_batches(sh)
    back.reorder_data(order)
    assert torch.equal(back["x"], d["x"]) and back["tags"] == d["tags"]
    sp, order = d.shard_by_batch_size(1, sequence_packing_args={"max_tokens_per_microbatch": 20,
                                                                "input_lengths_key": "lens"})
    assert sorted(order) == list(range(B))
    assert sum(m.size for m in sp[0].make_microbatch_iterator_for_packable_sequences()) == B
    rep = d.repeat_interleave(2)
    assert rep.size == 2 * B and rep["tags"][:2] == ["t0", "t0"]


# ---------------------------------------------------------------- packing
@pytest.mark.parametrize("alg", ["concatenative", "first_fit", "first_fit_decreasing", "first_fit_shuffle",
                                 "modified_first_fit_decreasing", "greedy_knapsack", "balanced_greedy_knapsack"])
def test_packers_valid(alg):
    from rl_b200.data.packing import get_packer

    rng = random.Random(0)
    lengths = [rng.randint(1, 100) for _ in range(200)]
    bins = get_packer(alg, bin_capacity=128).pack(lengths)
    seen = sorted(i for b in bins for i in b)
    assert seen == list(range(200))
    assert all(sum(lengths[i] for i in b) <= 128 for b in bins)
    lb = math.ceil(sum(lengths) / 128)
    if alg in ("modified_first_fit_decreasing", "first_fit_decreasing"):
        assert len(bins) <= math.ceil(1.25 * lb) + 1


# ----------------------------------------------------------------- losses
def _pg_data(B=3, S=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    tm = torch.ones(B, S)
    tm[:, 0] = 0
    tm[0, 4:] = 0
    return {"token_mask": tm, "sample_mask": torch.ones(B), "advantages": torch.randn(B, S, generator=g),
            "prev_logprobs": -torch.rand(B, S, generator=g), "generation_logprobs": -torch.rand(B, S, generator=g),
            "reference_policy_logprobs": -torch.rand(B, S, generator=g)}


def test_clipped_pg_matches_formula():
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn

    d = _pg_data()
    curr = (-torch.rand(3, 5)).requires_grad_(True)
    fn = ClippedPGLossFn({"ratio_clip_min": 0.2, "ratio_clip_max": 0.28, "reference_policy_kl_penalty": 0.0})
    gtok = d["token_mask"][:, 1:].sum()
    loss, m = fn(curr, d, torch.tensor(3.0), gtok)
    A = d["advantages"][:, 1:]
    r = torch.exp(curr - d["prev_logprobs"][:, 1:])
    per = torch.maximum(-A * r, -A * r.clamp(0.8, 1.28))
    mask = d["token_mask"][:, 1:]
    ref = (per * mask).sum() / (gtok + 1e-8)
    assert torch.allclose(loss, ref, atol=1e-6)
    loss.backward()
    assert curr.grad is not None and torch.isfinite(curr.grad).all()
    assert 0.8 - 1e-6 <= float(m["probs_ratio_clamped_min"]) <= float(m["probs_ratio_clamped_max"]) <= 1.28 + 1e-6


def test_kl_estimators_and_dual_clip_and_gspo():
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.algorithms.utils import calculate_kl

    a, b = torch.tensor([-1.0, -2.0]), torch.tensor([-1.5, -1.0])
    lr = b - a
    assert torch.allclose(calculate_kl(a, b, "k1"), -lr)
    assert torch.allclose(calculate_kl(a, b, "k2"), lr * lr / 2)
    assert torch.allclose(calculate_kl(a, b, "k3"), torch.exp(lr) - 1 - lr)
    d = _pg_data(seed=1)
    curr = -torch.rand(3, 5)
    for cfg in ({"ratio_clip_c": 3.0}, {"sequence_level_importance_ratios": True}, {"use_cispo": True},
                {"reference_policy_kl_penalty": 0.1, "reference_policy_kl_type": "k2"},
                {"use_importance_sampling_correction": True, "truncated_importance_sampling_type": "tis",
                 "truncated_importance_sampling_ratio": 2.0},
                {"use_importance_sampling_correction": True, "truncated_importance_sampling_type": "icepop",
                 "truncated_importance_sampling_ratio": 5.0, "truncated_importance_sampling_ratio_min": 0.5},
                {"disable_ppo_ratio": True}, {"force_on_policy_ratio": True}, {"token_level_loss": False},
                {"positive_example_nll_weight": 0.1}):
        loss, m = ClippedPGLossFn(cfg)(curr.clone().requires_grad_(True), d, torch.tensor(3.0),
                                       d["token_mask"][:, 1:].sum())
        assert torch.isfinite(loss), cfg


def test_dpo_nll_preference_losses():
    from rl_b200.algorithms.loss.loss_functions import DPOLossFn, NLLLossFn, PreferenceLossFn

    B, S = 4, 5
    tm = torch.ones(B, S)
    d = {"token_mask": tm, "sample_mask": torch.ones(B), "reference_policy_logprobs": torch.zeros(B, S),
         "input_lengths": torch.full((B,), S)}
    lp = torch.zeros(B, S - 1, requires_grad=True)
    loss, m = DPOLossFn({"reference_policy_kl_penalty": 0.1})(lp, d, torch.tensor(4.0), tm[:, 1:].sum())
    assert abs(float(loss) - math.log(2)) < 1e-5
    loss, _ = NLLLossFn()(torch.full((B, S - 1), -2.0), d, torch.tensor(4.0), tm[:, 1:].sum())
    assert abs(float(loss) - 2.0) < 1e-6
    r = torch.tensor([1.0, 0.0, 2.0, 3.0])
    loss, m = PreferenceLossFn()(r, d, torch.tensor(4.0), None)
    ref = -(torch.nn.functional.logsigmoid(torch.tensor(1.0)) + torch.nn.functional.logsigmoid(torch.tensor(-1.0))) / 2
    assert abs(float(loss) - float(ref)) < 1e-5


# ------------------------------------------------------ advantages
def _loo_reference(groups, rewards, valid):
    """Explicit per-group leave-one-out baseline / unbiased std."""
    B = len(rewards)
    base, std = torch.zeros(B), torch.zeros(B)
    for i in range(B):
        same = [j for j in range(B) if groups[j] == groups[i] and valid[j]]
        others = [j for j in same if j != i]
        if len(same) <= 1:
            base[i] = rewards[i]
            continue
        vals = torch.tensor([rewards[j] for j in others])
        base[i] = vals.mean()
        std[i] = vals.std(unbiased=True) if len(vals) > 1 else 0.0
    return base, std


def test_grpo_advantage_leave_one_out():
    from rl_b200.algorithms.advantage_estimator import GRPOAdvantageEstimator
    from rl_b200.algorithms.utils import calculate_baseline_and_std_per_prompt

    g = torch.Generator().manual_seed(0)
    groups = torch.tensor([0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2])
    rewards = torch.rand(12, generator=g)
    rewards[8:] = 0.5  # trivial group
    valid = torch.ones(12)
    base, std, trivial = calculate_baseline_and_std_per_prompt(groups, rewards, valid, True)
    rb, rs = _loo_reference(groups.tolist(), rewards.tolist(), valid.tolist())
    assert torch.allclose(base, rb, atol=1e-6)
    assert torch.allclose(std, rs, atol=1e-5)
    assert trivial[8:].all() and not trivial[:8].any()
    adv = GRPOAdvantageEstimator({}).compute_advantage(groups.view(-1, 1), rewards, torch.ones(12, 3))
    assert adv.shape == (12, 3)
    assert torch.allclose(adv[8:], torch.zeros(4, 3))
    assert torch.allclose(adv[:8, 0], (rewards[:8] - rb[:8]) / (rs[:8] + 1e-6), atol=1e-5)


def test_other_advantage_estimators():
    from rl_b200.algorithms.advantage_estimator import (GDPOAdvantageEstimator, GeneralizedAdvantageEstimator,
                                                        OPDAdvantageEstimator, ReinforcePlusPlusAdvantageEstimator)

    groups = torch.tensor([0, 0, 1, 1])
    mask = torch.ones(4, 3)
    batch = {"reward/a": torch.tensor([1.0, 0.0, 1.0, 1.0]), "reward/b": torch.tensor([0.0, 1.0, 0.5, 0.0])}
    adv = GDPOAdvantageEstimator({}).compute_advantage(groups, None, mask, repeated_batch=batch)
    assert adv.shape == (4, 3) and torch.isfinite(adv).all()
    adv = ReinforcePlusPlusAdvantageEstimator({}).compute_advantage(groups, torch.tensor([1.0, 0.0, 0.5, 0.2]), mask)
    assert abs(float((adv * mask).sum())) < 1e-4
    # GAE with lambda=1, gamma=1 and zero values: advantage = terminal reward at every valid token
    est = GeneralizedAdvantageEstimator({"gae_lambda": 1.0, "gae_gamma": 1.0, "normalize_advantages": False})
    adv, ret = est.compute_advantage(groups, torch.tensor([1.0, 2.0, 0.0, -1.0]), mask, values=torch.zeros(4, 3))
    assert torch.allclose(adv[:, 0], torch.tensor([1.0, 2.0, 0.0, -1.0]))
    opd = OPDAdvantageEstimator({})
    a = opd.compute_advantage(None, None, mask, logprobs_policy=torch.zeros(4, 3), logprobs_teacher=-torch.ones(4, 3))
    assert torch.allclose(a, -mask)


# ------------------------------------------------------------ checkpoints
def test_safetensors_roundtrip_and_hf_export(tmp_path):
    from rl_b200.models.checkpoint_io import hf_state_dict, load_hf_checkpoint, load_safetensors, save_hf_checkpoint, \
        save_safetensors
    from rl_b200.models.config import get_model_config
    from rl_b200.models.transformer import TransformerLM

    t = {"a": torch.randn(3, 4), "b": torch.arange(5, dtype=torch.int64), "c": torch.randn(2, 2).to(torch.bfloat16)}
    p = str(tmp_path / "x.safetensors")
    save_safetensors(t, p, {"format": "pt"})
    back = load_safetensors(p)
    for k in t:
        assert torch.equal(back[k], t[k])
    try:  # files written here are readable by the reference implementation of the format
        from safetensors.torch import load_file

        lib = load_file(p)
        assert torch.equal(lib["a"], t["a"])
    except ImportError:
        pass
    cfg = get_model_config("tiny-moe")
    m = TransformerLM(cfg, device="cpu", dtype=torch.float32, seed=1)
    sd = hf_state_dict(m, dtype=None)
    assert "model.layers.0.self_attn.q_proj.weight" in sd
    assert "model.layers.1.mlp.experts.7.down_proj.weight" in sd
    save_hf_checkpoint(m, str(tmp_path / "hf"))
    m2 = TransformerLM(cfg, device="cpu", dtype=torch.float32, seed=2)
    load_hf_checkpoint(m2, str(tmp_path / "hf"))
    # bf16 round trip of the saved copy
    assert torch.allclose(m2.flat_param, m.flat_param.to(torch.bfloat16).float())


def test_checkpoint_manager_topk_and_resume(tmp_path):
    from rl_b200.utils.checkpoint import CheckpointManager

    ck = CheckpointManager({"checkpoint_dir": str(tmp_path), "keep_top_k": 2, "metric_name": "train:loss",
                            "higher_is_better": False, "save_period": 1})
    for step, loss in [(1, 3.0), (2, 1.0), (3, 2.0), (4, 5.0)]:
        tmp = ck.init_tmp_checkpoint(step, {"current_step": step, "train": {"loss": loss}}, {"a": 1})
        ck.finalize_checkpoint(tmp)
    assert ck.list_steps() == [2, 3, 4]  # best two by loss (2, 3) + latest (4)
    assert ck.get_best_checkpoint_path().endswith("step_2")
    assert ck.load_training_info(ck.get_latest_checkpoint_path())["current_step"] == 4
    assert not any(n.startswith("tmp_") for n in os.listdir(tmp_path))


def test_policy_checkpoint_roundtrip_both_formats(tmp_path):
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY, _pcfg, make_batch
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn

    for fmt in ("safetensors", "torch_dist"):
        w = PolicyWorker(_pcfg(False), model_cfg=TINY, seed=3)
        w.train(make_batch(), ClippedPGLossFn({}), gbs=8)
        w.save_checkpoint(str(tmp_path / fmt / "w"), str(tmp_path / fmt / "o"), fmt=fmt)
        w2 = PolicyWorker(_pcfg(False), model_cfg=TINY, seed=9)
        w2.load_checkpoint(str(tmp_path / fmt / "w"), str(tmp_path / fmt / "o"))
        tol = 1e-2 if fmt == "safetensors" else 0.0  # safetensors export is bf16
        assert (w2.model.flat_param - w.model.flat_param).abs().max() <= tol + 1e-7
        assert w2.optimizer.step_count == w.optimizer.step_count


# ----------------------------------------------------------- environments
def test_environments():
    from rl_b200.environments.math_environment import MathEnvironment, answers_match, extract_answer
    from rl_b200.environments.registry import make_environment
    from rl_b200.environments.synthetic import EvenTokenEnvironment, hash_reward

    assert extract_answer("so the answer is \\boxed{\\frac{1}{2}}") == "\\frac{1}{2}"
    assert answers_match("1/2", "0.5") and answers_match("\\frac{1}{2}", "1/2") and not answers_match("3", "4")
    env = MathEnvironment()
    r = env.step([[{"role": "assistant", "content": "x = \\boxed{4}"}]], [{"ground_truth": "4"}])
    assert float(r.rewards[0]) == 1.0
    e = EvenTokenEnvironment().step([[{"role": "assistant", "token_ids": torch.tensor([2, 4, 5, 7])}]], [None])
    assert float(e.rewards[0]) == 0.5
    assert hash_reward(torch.tensor([1, 2, 3])) in (0.0, 1.0)
    code = make_environment("code", {"timeout_s": 10})
    ok = code.step([[{"role": "assistant", "content": "```python\ndef f(x):\n    return x + 1\n```"}]],
                   [{"tests": "assert f(1) == 2"}])
    assert float(ok.rewards[0]) == 1.0
    pz = make_environment("sliding_puzzle", {})
    res = pz.step([[{"role": "assistant", "content": "right"}]], [{"board": [[1, 2], [0, 3]]}])
    assert float(res.rewards[0]) == 1.0 and bool(res.terminateds[0])


# ---------------------------------------------------------- training loops
def _tiny_policy(seed=0, **kw):
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY

    cfg = {"max_total_sequence_length": 48, "precision": "float32", "train_global_batch_size": 8,
           "optimizer": {"kwargs": {"lr": 1e-3, "weight_decay": 0.0}},
           "generation": {"temperature": 1.0, "max_new_tokens": 8},
           "sequence_packing": {"train_mb_tokens": 96, "logprob_mb_tokens": 96}}
    cfg.update(kw)
    return PolicyWorker(cfg, model_cfg=TINY, seed=seed)


def test_grpo_tiny_config1_runs():
    from examples.run_grpo import main

    state = main(["--config", os.path.join(ROOT, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  "logger.log_dir=/tmp/rlb_test_logs", "logger.stdout=false"])
    assert state["current_step"] == 2


def test_sft_loss_decreases():
    from rl_b200.algorithms.sft import sft_train
    from rl_b200.data.datasets import SFTDataset, StatefulDataLoader

    g = random.Random(0)
    samples = [([g.randrange(512) for _ in range(6)], [7, 8, 9, 10, 11, 12]) for _ in range(16)]
    dl = StatefulDataLoader(SFTDataset(samples), 8, shuffle=False)
    w = _tiny_policy()
    losses = []
    sft_train(w, dl, {"sft": {"max_num_epochs": 6}, "policy": {"train_global_batch_size": 8}},
              step_callback=lambda s, m: losses.append(m["loss"]))
    assert len(losses) == 12 and losses[-1] < losses[0]


def test_sft_trains_on_packed_megatron_rows(tmp_path):
    from rl_b200.algorithms.sft import build_sft_batch, sft_train
    from rl_b200.data.datasets import StatefulDataLoader
    from rl_b200.data.response_datasets import load_response_dataset
    from rl_b200.data.tokenizer import get_tokenizer

    tok = get_tokenizer({"name": "byte"})
    path = tmp_path / "p.jsonl.packed"
    with open(path, "w") as f:
        for i in range(8):
            rec = [{"role": "system", "content": "s"}, {"role": "user", "content": f"u{i}"},
                   {"role": "assistant", "content": "abc"}, {"role": "system", "content": "t"},
                   {"role": "user", "content": "v"}, {"role": "assistant", "content": f"d{i}"}]
            f.write(json.dumps({"conv": rec}) + "\n")
    ds = load_response_dataset({"dataset_name": "megatron_sft_packed", "data_path": str(path), "chat_key": "conv",
                                "megatron_sft": {"prompt_format": "identity"}}, context_parallel_size=1)
    rows = [ds.processor(ds.dataset[i], ds.task_spec, tok, 24, i) for i in range(len(ds.dataset))]
    dl = StatefulDataLoader(rows, 4, shuffle=False)
    data = build_sft_batch(next(iter(dl)))
    assert data["input_ids"].shape[0] == 8  # two conversations per packed row
    assert float(data["token_mask"].sum()) == 4 * 9  # 10 text tokens a pack: 9 targets, padding masked
    w = _tiny_policy()
    losses = []
    sft_train(w, StatefulDataLoader(rows, 4, shuffle=False), {"sft": {"max_num_epochs": 5},
                                                              "policy": {"train_global_batch_size": 8}},
              step_callback=lambda s, m: losses.append(m["loss"]))
    assert len(losses) == 10 and losses[-1] < losses[0]


def test_preference_datasets_feed_the_dpo_loop(tmp_path):
    from rl_b200.algorithms.dpo import dpo_train
    from rl_b200.data.datasets import StatefulDataLoader
    from rl_b200.data.preference_datasets import PreferenceSamples, load_preference_dataset
    from rl_b200.data.tokenizer import get_tokenizer

    def jsonl(name, rows):
        with open(tmp_path / name, "w") as f:
            f.writelines(json.dumps(r) + "\n" for r in rows)
        return str(tmp_path / name)

    tok = get_tokenizer({"name": "byte"})
    b = jsonl("bin.jsonl", [{"q": f"p{i}", "good": "yes", "bad": "no!"} for i in range(8)])
    ds = load_preference_dataset({"dataset_name": "BinaryPreferenceDataset", "data_path": b, "prompt_key": "q",
                                  "chosen_key": "good", "rejected_key": "bad"})
    row = ds.dataset[0]
    assert row["context"] == [{"role": "user", "content": "p0"}] and row["completions"][0]["rank"] == 0
    smp = PreferenceSamples(ds, tok, 64)
    s0 = smp[0]
    assert tok.decode(s0["chosen"]).strip().endswith("yes") and tok.decode(s0["rejected"]).strip().endswith("no!")
    assert "p0" in tok.decode(s0["prompt"]) and "yes" not in tok.decode(s0["prompt"])
    # HelpSteer3 preference: the sign of overall_preference picks the side; 0 warns
    h = jsonl("hs.jsonl", [{"context": "c", "response1": "r1", "response2": "r2", "overall_preference": p}
                           for p in (-2, 3, 0)])
    ds = load_preference_dataset({"dataset_name": "HelpSteer3", "data_path": h})
    side = lambda r: [c["completion"][0]["content"] for c in sorted(r["completions"], key=lambda c: c["rank"])]
    assert side(ds.dataset[0]) == ["r1", "r2"] and side(ds.dataset[1]) == ["r2", "r1"]
    with pytest.warns(UserWarning):
        assert side(ds.dataset[2]) == ["r1", "r1"]
    # Tulu3: shared context checked
    t = jsonl("tulu.jsonl", [{"chosen": [{"role": "user", "content": "u"}, {"role": "assistant", "content": "A"}],
                              "rejected": [{"role": "user", "content": "u"}, {"role": "assistant", "content": "B"}]},
                             {"chosen": [{"role": "user", "content": "u"}, {"role": "assistant", "content": "A"}],
                              "rejected": [{"role": "user", "content": "v"}, {"role": "assistant", "content": "B"}]}])
    ds = load_preference_dataset({"dataset_name": "Tulu3Preference", "data_path": t})
    assert side(ds.dataset[0]) == ["A", "B"] and ds.dataset[0]["context"] == [{"role": "user", "content": "u"}]
    with pytest.raises(ValueError):
        ds.dataset[1]
    # generic rows already in the context / completions form, then the DPO loop on the binary set
    g = jsonl("gen.jsonl", [ds.dataset[0]])
    assert load_preference_dataset({"dataset_name": "PreferenceDataset", "data_path": g}).dataset[0][
        "task_name"].endswith("-gen")  # parent directory + file name
    out = []
    dpo_train(_tiny_policy(), StatefulDataLoader(smp, 4, shuffle=False, collate_fn=lambda x: x),
              {"dpo": {"max_num_epochs": 1, "reference_policy_kl_penalty": 0.1}}, step_callback=lambda s, m: out.append(m))
    assert len(out) == 2 and all(math.isfinite(m["loss"]) for m in out)


def test_dpo_and_rm_loops():
    from rl_b200.algorithms.dpo import dpo_train, rm_train
    from rl_b200.data.datasets import PreferenceDataset, StatefulDataLoader

    g = random.Random(1)
    samples = [([g.randrange(512) for _ in range(5)], [1, 2, 3], [4, 5, 6, 7]) for _ in range(8)]
    dl = StatefulDataLoader(PreferenceDataset(samples), 4, shuffle=False, collate_fn=lambda b: b)
    out = []
    dpo_train(_tiny_policy(), dl, {"dpo": {"max_num_epochs": 2, "reference_policy_kl_penalty": 0.1}},
              step_callback=lambda s, m: out.append(m))
    assert len(out) == 4 and all(math.isfinite(m["loss"]) for m in out)
    rm = _tiny_policy(num_labels=1)
    out = []
    rm_train(rm, StatefulDataLoader(PreferenceDataset(samples), 4, shuffle=False, collate_fn=lambda b: b),
             {"rm": {"max_num_epochs": 3}}, step_callback=lambda s, m: out.append(m))
    assert len(out) == 6 and out[-1]["loss"] < out[0]["loss"] + 1e-6
    # MPO: DPO + SFT + BCO with a driver-side reward-shift EMA
    from rl_b200.algorithms.dpo import mpo_train

    out = []
    st = mpo_train(_tiny_policy(), StatefulDataLoader(PreferenceDataset(samples), 4, shuffle=False,
                                                      collate_fn=lambda b: b),
                   {"mpo": {"max_num_epochs": 1, "reference_policy_kl_penalty": 0.1, "sft_loss_weight": 0.5,
                            "bco_loss_weight": 1.0, "reward_shift_momentum": 0.5}},
                   step_callback=lambda s, m: out.append(m))
    assert len(out) == 2 and all(math.isfinite(m["loss"]) and "bco_loss" in m for m in out)
    assert "reward_shift" in st and math.isfinite(st["reward_shift"])


def test_ppo_and_distillation_loops():
    from rl_b200.algorithms.distillation import distillation_train, kd_train
    from rl_b200.algorithms.ppo import ppo_train
    from rl_b200.algorithms.sft import build_sft_batch
    from rl_b200.data.datasets import SFTDataset, StatefulDataLoader, SyntheticPromptDataset
    from rl_b200.environments.synthetic import EvenTokenEnvironment

    ds = SyntheticPromptDataset(16, 6, 10, 512, seed=0)
    env = {"synthetic": EvenTokenEnvironment()}
    cfg = {"ppo": {"num_generations_per_prompt": 2, "max_num_steps": 2}, "loss_fn": {},
           "policy": {"max_total_sequence_length": 48}}
    seen = []
    ppo_train(_tiny_policy(), _tiny_policy(seed=5, num_labels=1), StatefulDataLoader(ds, 4, shuffle=False), env, cfg,
              step_callback=lambda s, m: seen.append(m))
    assert len(seen) == 2 and all(math.isfinite(m["value_loss"]) for m in seen)
    seen = []
    distillation_train(_tiny_policy(), _tiny_policy(seed=11), StatefulDataLoader(ds, 4, shuffle=False), env,
                       {"distillation": {"max_num_steps": 2}, "policy": {"max_total_sequence_length": 48}},
                       step_callback=lambda s, m: seen.append(m))
    assert len(seen) == 2
    samples = [([1, 2, 3], [4, 5, 6]) for _ in range(4)]
    batches = [build_sft_batch(b) for b in StatefulDataLoader(SFTDataset(samples), 4, shuffle=False)]
    seen = []
    kd_train(_tiny_policy(), _tiny_policy(seed=3), batches, {"distillation": {}}, k=8,
             step_callback=lambda s, m: seen.append(m))
    assert len(seen) == 1 and math.isfinite(seen[0]["loss"])


def test_flops_formula_and_mfu():
    from rl_b200.models.config import get_model_config
    from rl_b200.utils.flops import FLOPTracker, forward_flops, mfu

    cfg = get_model_config("llama3.1-8b")
    # ~2 x 8.03e9 params per token (embedding lookup excluded, LM head included) + attention
    f = forward_flops(cfg, [1])
    n_lin = 32 * (4096 * (4096 + 2 * 1024) + 4096 * 4096 + 3 * 4096 * 14336) + 4096 * 128256
    assert abs(f - 2 * n_lin - 32 * 2 * 32 * 128) < 1
    tr = FLOPTracker(cfg)
    tr.track([1024, 512])
    assert tr.model_train_flops() == 3 * forward_flops(cfg, [1024, 512])
    assert abs(mfu(2250e12, 1.0, 1, device="B200") - 1.0) < 1e-9


def test_eval_pass_and_cons_at_k():
    from rl_b200.evals.eval import eval_cons_k, eval_pass_k

    r = torch.tensor([1.0, 0.0, 0.0, 0.0, 1.0, 1.0, 0.0, 0.0])
    # group 1: n=4, c=1 -> pass@2 = 1 - C(3,2)/C(4,2) = 0.5; group 2: c=2 -> 1 - C(2,2)/C(4,2) = 5/6
    assert abs(eval_pass_k(r, 4, 2) - (0.5 + 5 / 6)) < 1e-9
    assert eval_pass_k(r, 4, 4) == 2.0
    ans = ["a", "b", "b", "c", "x", "x", "y", "x"]
    r2 = torch.tensor([0.0, 1.0, 1.0, 0.0, 1.0, 1.0, 0.0, 1.0])
    # group 1: majority of all 4 is "b" (rewarded): cons@4 = 1; group 2: "x" rewarded -> 1
    assert eval_cons_k(r2, 4, 4, ans) == 2.0
    # cons@1 = mean reward of the group
    assert abs(eval_cons_k(r2, 4, 1, ans) - (0.5 + 0.75)) < 1e-9


def test_spec_verify_reference_distribution():
    from rl_b200.ops.spec_decode import spec_verify_ref

    g = torch.Generator().manual_seed(0)
    B, V, k = 4000, 4, 1
    t_row = torch.randn(k + 1, V, generator=g)
    d_row = torch.randn(k, V, generator=g)
    q = torch.softmax(d_row, -1)
    draft = torch.multinomial(q[0], B, replacement=True, generator=g).unsqueeze(1)
    tok, n, _ = spec_verify_ref(t_row.expand(B, k + 1, V), d_row.expand(B, k, V), draft, 1.0, g)
    freq = torch.bincount(tok[:, 0], minlength=V).float() / B
    assert (freq - torch.softmax(t_row[0], -1)).abs().max() < 0.03


def test_speculative_decoding_greedy_matches_plain_decoding():
    """Greedy speculative decoding (1-layer draft, 2 proposals per round) emits
    exactly the target's greedy continuation."""
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.transformer import TransformerLM
    from tests.dist_cases import TINY

    w = _tiny_policy(seed=2, generation={"temperature": 1.0, "max_new_tokens": 12,
                                         "mcore_generation_config": {"block_size_tokens": 8}})
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, TINY.vocab_size, (3, 10), generator=g)
    data = BatchedDataDict({"input_ids": ids, "input_lengths": torch.tensor([10, 7, 4])})
    ref = w.generate(data, greedy=True)
    draft = TransformerLM(TINY.replace(num_layers=1), w.ps, dtype=w.model.dtype, seed=11)
    w.engine.set_draft(draft, 2)
    out = w.generate(data, greedy=True)
    assert torch.equal(out["output_ids"], ref["output_ids"])
    assert torch.equal(out["generation_lengths"], ref["generation_lengths"])
    assert w.engine.spec_stats["rounds"] > 0
    # sampling mode runs end to end and stays within the budget
    out2 = w.generate(data)
    assert int(out2["generation_lengths"].max()) <= 12


def test_worker_speculative_config_and_draft_training():
    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    w = _tiny_policy(seed=2, generation={"temperature": 1.0, "max_new_tokens": 8,
                                         "speculative": {"num_speculative_tokens": 2, "draft_num_layers": 1},
                                         "mcore_generation_config": {"block_size_tokens": 8}})
    assert w.draft is not None and w.engine.num_spec == 2
    g = torch.Generator().manual_seed(5)
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (4, 12), generator=g),
                            "input_lengths": torch.tensor([12, 9, 5, 12])})
    out = w.generate(data)
    assert w.engine.spec_stats["rounds"] > 0
    seqs = BatchedDataDict({"input_ids": out["output_ids"], "input_lengths": out["unpadded_sequence_lengths"]})
    l0 = w.train_draft(seqs)
    for _ in range(10):
        l1 = w.train_draft(seqs)
    assert l1 < l0


def test_train_time_top_k_top_p_logprobs():
    """With top-k / top-p rollouts the trainer's log-probs are those of the
    filtered, renormalised distribution; TP=1 vs the explicit formula."""
    from rl_b200.ops.fused_linear_logprob import filter_logits_top_k_top_p, filtered_linear_logprobs

    g = torch.Generator().manual_seed(1)
    h = torch.randn(7, 16, generator=g)
    w = torch.randn(50, 16, generator=g)
    tgt = torch.randint(0, 50, (7,), generator=g)
    logits = h @ w.t()
    keep = logits.topk(5, -1).values[:, -1:]
    ref = torch.log_softmax(logits.masked_fill(logits < keep, float("-inf")), -1).gather(1, tgt[:, None]).squeeze(1)
    lp, _ = filtered_linear_logprobs(h, w, tgt, 0, 1.0, 5, 1.0)
    assert torch.allclose(lp, ref)
    # nucleus: the kept set is the smallest prefix of sorted probs whose mass reaches p
    x = torch.tensor([[3.0, 2.0, 1.0, 0.0]])
    out = filter_logits_top_k_top_p(x, None, 0.8)
    p = torch.softmax(x, -1)[0]
    n_keep = int((torch.cumsum(p, 0) - p < 0.8).sum())
    assert int(torch.isfinite(out).sum()) == n_keep


def test_numa_binding_from_fake_sysfs(tmp_path):
    from rl_b200.utils.numa import bind_to_gpu_numa, parse_cpulist

    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    dev = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    dev.mkdir(parents=True)
    before = os.sched_getaffinity(0)
    cpu = sorted(before)[0]
    (dev / "local_cpulist").write_text(f"{cpu}\n")
    try:
        used = bind_to_gpu_numa(sysfs_root=str(tmp_path), pci_bus_id="1b:00.0")
        assert used == [cpu] and os.sched_getaffinity(0) == {cpu}
        assert bind_to_gpu_numa(sysfs_root=str(tmp_path), pci_bus_id="ff:00.0") is None
    finally:
        os.sched_setaffinity(0, before)


def test_telemetry_spans_and_goodput(tmp_path):
    from rl_b200.utils.telemetry import Telemetry, read_otlp_spans

    t = Telemetry(str(tmp_path / "spans.jsonl"))
    with t.span("step", step=1):
        with t.span("generation"):
            pass
    g = t.goodput({"generation": 2.0, "policy_training": 3.0, "weight_sync": 0.5, "total_step_time": 6.0}, 6.0)
    assert abs(g["goodput/fraction"] - 5 / 6) < 1e-9 and abs(g["goodput/idle_s"] - 0.5) < 1e-9
    assert t.flush() == 2
    recs = {r["name"]: r for r in read_otlp_spans(str(tmp_path / "spans.jsonl"))}
    assert set(recs) == {"step", "generation"}
    assert recs["generation"]["parentSpanId"] == recs["step"]["spanId"]
    assert recs["generation"]["traceId"] == recs["step"]["traceId"]
    assert {"key": "rl.bucket", "value": {"stringValue": "productive"}} in recs["generation"]["attributes"]


def test_prev_logprobs_folded_into_training_forward():
    """One optimizer step per batch: taking prev_logprobs from the step's own
    forward equals the separate inference pass."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from tests.dist_cases import make_batch

    data = make_batch(B=8, S=24, seed=7)
    lf = ClippedPGLossFn({"reference_policy_kl_penalty": 0.0})
    a = _tiny_policy(seed=4)
    d1 = data.copy()
    d1["prev_logprobs"] = a.get_logprobs(d1)["logprobs"]
    ra = a.train(d1, lf, gbs=8)
    b = _tiny_policy(seed=4)
    d2 = data.copy()
    d2["prev_logprobs"] = torch.zeros_like(d2["prev_logprobs"])
    rb = b.train(d2, lf, gbs=8, prev_from_current=True)
    assert abs(ra["loss"] - rb["loss"]) < 1e-6 and abs(ra["grad_norm"] - rb["grad_norm"]) < 1e-5
    assert torch.allclose(a.model.flat_param, b.model.flat_param)


def test_fp8_rollout_weights_used_and_refreshed():
    """fp8 rollout (vllm_cfg.precision: fp8): the refit quantises the linear
    weights (128 x 128 blocks, power-of-two scales), the rollout forwards use
    them (close to the bf16 forward, not identical), training forwards do not,
    and a training step refreshes them."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import make_batch

    cfg = ModelConfig(name="tiny-128", vocab_size=512, hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=32, ffn_hidden_size=256, rope_theta=10000.0, max_position_embeddings=256)
    pc = {"max_total_sequence_length": 48, "precision": "float32", "train_global_batch_size": 8,
          "optimizer": {"kwargs": {"lr": 1e-2, "weight_decay": 0.0}},
          "generation": {"temperature": 1.0, "max_new_tokens": 6, "vllm_cfg": {"precision": "fp8"},
                         "mcore_generation_config": {"block_size_tokens": 8}},
          "sequence_packing": {"train_mb_tokens": 96, "logprob_mb_tokens": 96}}
    w = PolicyWorker(pc, model_cfg=cfg, seed=1)
    fw = w.gen_model.fp8_weights
    assert fw is not None and len(fw) == 4 * cfg.num_layers and w.gen_model.fp8_pow2
    name = "model.layers.0.mlp.down_proj.weight"
    q0 = fw[name][0].float().clone()
    x = torch.randn(5, 256)
    ref = x @ w.model.param(name).detach().t()
    w.gen_model._in_rollout = True
    y = w.gen_model._lin_infer(x, name)
    w.gen_model._in_rollout = False
    err = ((y.float() - ref).norm() / ref.norm()).item()
    assert 0 < err < 0.08
    assert torch.equal(w.gen_model._lin_infer(x, name), torch.nn.functional.linear(x, w.model.param(name)))
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (3, 9)), "input_lengths": torch.tensor([9, 5, 7])})
    out = w.generate(data)
    assert int(out["generation_lengths"].min()) >= 1
    b = make_batch(B=8, S=24, vocab=512)
    w.train(b, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=8)
    w.refit()
    assert not torch.equal(w.gen_model.fp8_weights[name][0].float(), q0)


def test_fp8_training_linear_and_loop():
    """fp8 blockwise training: fprop and dgrad through block-scaled e4m3 GEMMs
    (1x128 activations / gradients, 128x128 weights and their transpose), wgrad
    in full precision; the weight cache follows the model's weight version; a
    few GRPO-loss steps with fp8 on track the bf16/fp32 run."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.ops.fp8_linear import fp8_train_linear
    from tests.dist_cases import make_batch

    torch.manual_seed(0)
    for pow2 in (True, False):
        x = torch.randn(50, 256, requires_grad=True)
        w = torch.nn.Parameter(torch.randn(384, 256) * 0.05)
        cache = {}
        y = fp8_train_linear(x, w, cache, "w", 0, pow2)
        g = torch.randn_like(y)
        (y * g).sum().backward()
        x2 = x.detach().clone().requires_grad_(True)
        w2 = w.detach().clone().requires_grad_(True)
        y2 = x2 @ w2.t()
        (y2 * g).sum().backward()
        rel = lambda a, b: ((a - b).norm() / b.norm()).item()  # noqa: E731
        assert rel(y.float(), y2) < 0.08 and rel(x.grad, x2.grad) < 0.08
        assert torch.allclose(w.grad, w2.grad, atol=1e-4)  # wgrad is not quantised
        fw = cache["w"]
        fp8_train_linear(x, w, cache, "w", 0, pow2)
        assert cache["w"] is fw  # same version: cached
        fp8_train_linear(x, w, cache, "w", 1, pow2)
        assert cache["w"] is not fw

    cfg = ModelConfig(name="tiny-128", vocab_size=512, hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=32, ffn_hidden_size=256, rope_theta=10000.0, max_position_embeddings=256)

    def run(fp8):
        pc = {"max_total_sequence_length": 48, "precision": "float32", "train_global_batch_size": 8,
              "optimizer": {"kwargs": {"lr": 3e-3, "weight_decay": 0.0}},
              "megatron_cfg": {"fp8_cfg": {"enabled": fp8, "fp8": "e4m3", "fp8_recipe": "blockwise"}},
              "generation": {"temperature": 1.0, "max_new_tokens": 4},
              "sequence_packing": {"train_mb_tokens": 96, "logprob_mb_tokens": 96}}
        w = PolicyWorker(pc, model_cfg=cfg, seed=1)
        b = make_batch(B=8, S=24, vocab=512)
        losses = [w.train(b, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=8)["loss"]
                  for _ in range(3)]
        return losses, w

    l8, w8 = run(True)
    l32, _ = run(False)
    assert w8.model.fp8_train is not None and len(w8.model._fp8_cache) == 4 * cfg.num_layers
    assert w8.model.weight_version == 3
    assert all(abs(a - b) < 0.05 * max(1.0, abs(b)) for a, b in zip(l8, l32)), (l8, l32)


def test_quantization_aware_training():
    """Fake-quantised training (policy.quant_cfg): fp8 block / per-tensor and
    NVFP4 quantise-dequantise match their definitions, gradients pass straight
    through, calibration records input amax, and QAT training runs."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.models.quantization import E2M1_VALUES, QATConfig, QuantSpec, fake_quant
    from rl_b200.ops.quant import dequant_fp8_block, quant_fp8_block_ref
    from tests.dist_cases import make_batch

    torch.manual_seed(0)
    w = torch.randn(200, 300)
    q, s = quant_fp8_block_ref(w, 128)
    assert torch.allclose(fake_quant(w, QuantSpec("fp8", (128, 128))), dequant_fp8_block(q, s), atol=1e-6)
    x = torch.randn(7, 64)
    f4 = fake_quant(x, QuantSpec("nvfp4", (1, 16)))
    # every 16-block is (e4m3 block scale) x (e2m1 values)
    blk = f4.view(7, 4, 16)
    sc = blk.abs().amax(-1, keepdim=True) / 6.0
    vals = (blk / sc.clamp_min(1e-30)).abs()
    assert torch.isin(vals.round(decimals=4), E2M1_VALUES.round(decimals=4)).float().mean() > 0.99
    assert ((f4 - x).norm() / x.norm()).item() < 0.2
    cfg = ModelConfig(name="tiny-128", vocab_size=512, hidden_size=128, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=32, ffn_hidden_size=256, rope_theta=10000.0, max_position_embeddings=256)
    assert QATConfig.from_cfg("NVFP4_W4A16_CFG").input is None
    for preset in ("FP8_BLOCK_CFG", "FP8_DEFAULT_CFG", "NVFP4_DEFAULT_CFG"):
        pc = {"max_total_sequence_length": 48, "precision": "float32", "train_global_batch_size": 8,
              "optimizer": {"kwargs": {"lr": 3e-3, "weight_decay": 0.0}}, "quant_cfg": preset,
              "generation": {"temperature": 1.0, "max_new_tokens": 4},
              "sequence_packing": {"train_mb_tokens": 96, "logprob_mb_tokens": 96}}
        wk = PolicyWorker(pc, model_cfg=cfg, seed=1)
        b = make_batch(B=8, S=24, vocab=512)
        stats = wk.calibrate_quantizers(b)
        assert len(stats) == 4 * cfg.num_layers and all(v > 0 for v in stats.values())
        assert not any("lm_head" in k or "embed" in k for k in stats)
        p0 = wk.model.param("model.layers.0.mlp.down_proj.weight").detach().clone()
        res = wk.train(b, ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}), gbs=8)
        assert res["grad_norm"] > 0
        assert not torch.equal(wk.model.param("model.layers.0.mlp.down_proj.weight"), p0)


def test_fp8_kv_cache_calibration():
    """fp8 KV cache (vllm_cfg.kv_cache_dtype: fp8) with per-layer scales from
    calibrate_qkv_fp8_scales: the cache stores k / k_scale in e4m3 and the
    rollout log-probs stay close to the trainer's."""
    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    w = _tiny_policy(seed=3, generation={"temperature": 1.0, "max_new_tokens": 8,
                                         "vllm_cfg": {"kv_cache_dtype": "fp8"},
                                         "mcore_generation_config": {"block_size_tokens": 8}})
    assert w.engine.kv_dtype == torch.float8_e4m3fn
    g = torch.Generator().manual_seed(4)
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (4, 12), generator=g),
                            "input_lengths": torch.tensor([12, 9, 6, 10])})
    sc = w.calibrate_qkv_fp8_scales(data)
    assert len(sc) == 2 and all(v["k_scale"] > 0 and v["v_scale"] > 0 for v in sc.values())
    out = w.generate(data)
    assert w.engine.kv.k_scales == [sc[f"layer_{i}"]["k_scale"] for i in range(2)]
    seqs = BatchedDataDict({"input_ids": out["output_ids"], "input_lengths": out["unpadded_sequence_lengths"]})
    lp = w.get_logprobs(seqs)["logprobs"]
    mask = torch.zeros_like(lp, dtype=torch.bool)
    for b in range(4):
        L, n = int(data["input_lengths"][b]), int(out["generation_lengths"][b])
        mask[b, L:L + n] = True
    assert (lp - out["logprobs"])[mask].abs().mean().item() < 0.1


def test_policy_facade():
    """The reference-style Policy facade forwards to the local worker."""
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.policy.lm_policy import Policy

    w = _tiny_policy(seed=4)
    pol = Policy(w)
    g = torch.Generator().manual_seed(1)
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (3, 10), generator=g),
                            "input_lengths": torch.tensor([10, 6, 8])})
    lp = pol.get_logprobs(data)["logprobs"]
    tk = pol.get_topk_logits(data, k=4)
    assert tk["topk_logits"].shape == (3, 10, 4)
    # the target token's logprob equals its logit minus logsumexp; top-1 >= every other
    assert (tk["topk_logits"][:, :, 0] >= tk["topk_logits"][:, :, 1]).all()
    assert pol.data_parallel_size == 1 and pol.prepare_for_generation()
    out = pol.generate(data, greedy=True)
    assert out["output_ids"].shape[0] == 3
    info = pol.prepare_refit_info()
    assert "model.embed_tokens.weight" in info
    assert torch.equal(pol.run_all_workers_single_data("get_logprobs", data)["logprobs"], lp)
    assert pol.shutdown()


def test_kl_uses_unfiltered_logprobs_under_top_k():
    """With train-time top-k filtering and a KL penalty, the loss receives the
    unfiltered current log-probs for its KL term (they differ from the
    filtered ones)."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from tests.dist_cases import make_batch

    w = _tiny_policy(seed=6, generation={"temperature": 1.0, "top_k": 8, "max_new_tokens": 4})
    seen = {}
    base = ClippedPGLossFn({"reference_policy_kl_penalty": 0.1})

    def spy(curr, mb, gs, gt):
        seen["unf"] = mb.get("curr_logprobs_unfiltered")
        seen["curr"] = curr.detach()
        return base(curr, mb, gs, gt)

    spy.kl_coef = base.kl_coef
    b = make_batch(B=4, S=16, vocab=512)
    b["reference_policy_logprobs"] = b["prev_logprobs"].clone()
    w.train(b, spy, gbs=4)
    assert seen["unf"] is not None
    m = b["token_mask"][:, 1:].bool()[:, :seen["curr"].shape[1]]
    c, u = seen["curr"][m], seen["unf"][m]
    assert torch.isfinite(u).all() and not torch.allclose(c, u)
    # kept tokens: the filter renormalises over 8 tokens, so their log-probs are higher
    kept = torch.isfinite(c) & (c > -1e8)
    assert (c[kept] >= u[kept] - 1e-5).all()


def test_opd_trust_region_advantages():
    """On-policy distillation advantages: plain OPD at alpha = 1, trust-region
    mixture below it (bounded by log(1 - alpha)), global baseline over valid
    tokens only, metrics on the raw teacher-student gap; the reference's keyword
    names are accepted."""
    import pytest

    from rl_b200.algorithms.advantage_estimator import OPDAdvantageEstimator

    teacher = torch.tensor([[-0.2, -1.7, -0.5]])
    student = torch.tensor([[-1.2, -0.8, -0.5]])
    ones = torch.ones_like(teacher)
    plain = OPDAdvantageEstimator({"proximal_teacher_alpha": 1.0})
    torch.testing.assert_close(plain.compute_advantage(None, None, ones, teacher_logprobs=teacher,
                                                       prev_logprobs=student), teacher - student)
    a = 0.2
    tr = OPDAdvantageEstimator({"proximal_teacher_alpha": a})
    exp = torch.log(a * torch.exp(teacher) + (1 - a) * torch.exp(student)) - student
    torch.testing.assert_close(tr.compute_advantage(None, None, ones, teacher_logprobs=teacher,
                                                    prev_logprobs=student), exp)
    low = tr.compute_advantage(None, None, ones, teacher_logprobs=torch.full((1, 3), -80.0),
                               prev_logprobs=torch.tensor([[-0.1, -1.0, -3.0]]))
    torch.testing.assert_close(low, torch.full_like(low, math.log1p(-a)))
    # global baseline: the masked position neither votes nor receives advantage
    t2 = torch.tensor([[0.0, -1.0], [-2.0, -0.5]])
    s2 = torch.tensor([[-1.0, -1.0], [-1.0, -3.0]])
    m2 = torch.tensor([[1.0, 1.0], [0.0, 1.0]])
    g = OPDAdvantageEstimator({"subtract_global_baseline": True})
    torch.testing.assert_close(g.compute_advantage(None, None, m2, teacher_logprobs=t2, prev_logprobs=s2),
                               (t2 - s2 - 7.0 / 6.0) * m2)
    m3 = torch.tensor([[1.0, 1.0, 0.0]])
    est = OPDAdvantageEstimator({"proximal_teacher_alpha": 0.2})
    adv = est.compute_advantage(None, None, m3, teacher_logprobs=torch.tensor([[0.0, -1.0, 5.0]]),
                                prev_logprobs=torch.tensor([[-1.0, -1.0, -5.0]]))
    assert est.last_metrics["on_policy_distillation/teacher_student_logprob_gap_mean"] == pytest.approx(0.5)
    assert est.last_metrics["on_policy_distillation/adv_mean"] == pytest.approx(adv[:, :2].mean().item())
    allm = OPDAdvantageEstimator({"proximal_teacher_alpha": 0.2, "subtract_global_baseline": True})
    z = allm.compute_advantage(None, None, torch.zeros(1, 3), teacher_logprobs=torch.zeros(1, 3),
                               prev_logprobs=torch.zeros(1, 3))
    assert torch.isfinite(z).all() and (z == 0).all()
    for bad in (0.0, -0.1, 1.01):
        with pytest.raises(ValueError):
            OPDAdvantageEstimator({"proximal_teacher_alpha": bad})


def test_reward_shaping_and_scaling_semantics():
    """DAPO overlong penalty (linear, uncapped), stop-properly penalty for
    truncated samples, required settings, and linear reward scaling with clipping
    (the reference's documented examples)."""
    import pytest

    from rl_b200.algorithms.grpo import apply_reward_shaping, scale_rewards

    cfg = {"enabled": True, "overlong_buffer_length": 5, "overlong_buffer_penalty": 0.5, "max_response_length": 25}
    out = apply_reward_shaping(torch.tensor([1.0, 0.8, 0.6, 0.4]), torch.tensor([10, 22, 25, 30]), cfg)
    torch.testing.assert_close(out, torch.tensor([1.0, 0.6, 0.1, -0.6]))
    same = apply_reward_shaping(torch.tensor([1.0, 0.5, 0.8]), torch.tensor([10, 15, 18]),
                                dict(cfg, overlong_buffer_penalty=1.0))
    torch.testing.assert_close(same, torch.tensor([1.0, 0.5, 0.8]))
    sp = apply_reward_shaping(torch.tensor([1.0, 0.8, 0.6, 0.4]), torch.tensor([10, 20, 30, 40]),
                              {"enabled": True, "stop_properly_penalty_coef": 0.5},
                              truncated=torch.tensor([False, True, False, True]))
    torch.testing.assert_close(sp, torch.tensor([1.0, 0.4, 0.6, 0.2]))
    with pytest.raises(ValueError, match="DAPO reward shaping"):
        apply_reward_shaping(torch.ones(1), torch.tensor([20]), {"enabled": True, "overlong_buffer_penalty": 0.1,
                                                                 "max_response_length": 25})
    with pytest.raises(AssertionError, match="stop_properly_penalty_coef must be in"):
        apply_reward_shaping(torch.ones(2), torch.tensor([1, 2]), {"enabled": True, "stop_properly_penalty_coef": 1.5},
                             truncated=torch.tensor([False, True]))
    sc = scale_rewards(torch.tensor([-2.8, -0.25, 1.5, 0.5, 2.0, 2.5]),
                       {"enabled": True, "source_min": -2.0, "source_max": 2.0, "target_min": -1.0, "target_max": 1.0})
    torch.testing.assert_close(sc, torch.tensor([-1.0, -0.125, 0.75, 0.25, 1.0, 1.0]))


def test_dynamic_sampling_and_masked_reward_policy():
    """Dynamic sampling keeps a mixed group entire (judged on the whole group,
    not leave-one-out peers) and, under masked_reward_policy "exclude", only
    rows with a loss weight vote; the GRPO baseline ignores invalid rows."""
    from rl_b200.algorithms.advantage_estimator import GRPOAdvantageEstimator
    from rl_b200.algorithms.grpo import dynamic_sampling

    keep = dynamic_sampling(torch.tensor([0.0] + [0.95] * 7 + [1.0] * 4), torch.tensor([0] * 8 + [1] * 4))
    assert keep.tolist() == [True] * 8 + [False] * 4
    r, g = torch.tensor([1.0, 1.0, 1.0, 0.0]), torch.zeros(4, dtype=torch.long)
    assert dynamic_sampling(r, g).all()
    assert not dynamic_sampling(r, g, torch.tensor([1.0, 1.0, 1.0, 0.0])).any()
    est = GRPOAdvantageEstimator({"use_leave_one_out_baseline": False, "normalize_rewards": False})
    adv = est.compute_advantage(torch.zeros(4, 3, dtype=torch.long), torch.tensor([1.0, 3.0, 2.0, 0.0]),
                                torch.ones(4, 5), valid_mask=torch.tensor([1.0, 1.0, 1.0, 0.0]))
    torch.testing.assert_close(adv[:3, 0], torch.tensor([-1.0, 1.0, 0.0]))


def test_message_level_advantage_penalties():
    """Flagged assistant messages get the configured advantage on their tokens;
    flagged user messages and unflagged tokens keep theirs; broadcast advantages
    are materialised (the reference's documented examples)."""
    from rl_b200.algorithms.grpo import apply_message_level_advantage_penalties
    from rl_b200.distributed.batched_data_dict import BatchedDataDict

    td = BatchedDataDict({"advantages": torch.tensor([[0.0, 1, 2, 3, 4, 5], [10.0, 11, 12, 13, 14, 15]])})
    logs = [[{"role": "user", "token_ids": torch.tensor([1, 2]), "is_invalid_tool_call": True},
             {"role": "assistant", "token_ids": torch.tensor([3, 4]), "is_invalid_tool_call": True},
             {"role": "assistant", "token_ids": torch.tensor([5, 6])}],
            [{"role": "user", "token_ids": torch.tensor([7])},
             {"role": "assistant", "token_ids": torch.tensor([8, 9, 10]), "has_malformed_thinking": True},
             {"role": "assistant", "token_ids": torch.tensor([11, 12])}]]
    apply_message_level_advantage_penalties(td, logs, -5.0, -7.0)
    torch.testing.assert_close(td["advantages"], torch.tensor([[0.0, 1, -5, -5, 4, 5], [10.0, -7, -7, -7, 14, 15]]))
    per = torch.tensor([[1.0], [10.0]])
    td2 = BatchedDataDict({"advantages": per.expand(2, 6)})
    logs2 = [[{"role": "user", "token_ids": torch.tensor([1])},
              {"role": "assistant", "token_ids": torch.tensor([2, 3, 4]), "is_invalid_tool_call": True},
              {"role": "assistant", "token_ids": torch.tensor([5, 6])}],
             [{"role": "user", "token_ids": torch.tensor([7, 8])},
              {"role": "assistant", "token_ids": torch.tensor([9, 10]), "has_malformed_thinking": True},
              {"role": "assistant", "token_ids": torch.tensor([11, 12])}]]
    apply_message_level_advantage_penalties(td2, logs2, -5.0, -7.0)
    torch.testing.assert_close(td2["advantages"], torch.tensor([[1.0, -5, -5, -5, 1, 1], [10.0, 10, -7, -7, 10, 10]]))
    torch.testing.assert_close(per, torch.tensor([[1.0], [10.0]]))


def test_training_stops_and_saves_before_deadline(tmp_path):
    """checkpoint_must_save_by: when the next step would cross the deadline the
    loop saves a checkpoint and stops early (the save period alone would not)."""
    from rl_b200.algorithms.sft import sft_train
    from rl_b200.data.datasets import SFTDataset, StatefulDataLoader
    from rl_b200.utils.checkpoint import CheckpointManager

    w = _tiny_policy(seed=3)
    g = random.Random(1)
    samples = [([g.randrange(512) for _ in range(6)], [7, 8, 9, 10]) for _ in range(400)]
    dl = StatefulDataLoader(SFTDataset(samples), 8, shuffle=False)
    ck = CheckpointManager({"enabled": True, "checkpoint_dir": str(tmp_path), "save_period": 1000,
                            "checkpoint_must_save_by": "00:00:00:01"})
    import time

    state = sft_train(w, dl, {"sft": {"max_num_steps": 50, "val_period": 0},
                              "policy": {"train_global_batch_size": 8}},
                      checkpointer=ck, step_callback=lambda s, m: time.sleep(0.3))
    assert 1 <= state["current_step"] < 50
    assert ck.list_steps() == [state["current_step"]]


def test_overlapped_reduction_bookkeeping():
    """overlap_grad_reduce bookkeeping: ``step`` reduces exactly the parts of the
    shard that no completed layer bucket covered; setup is refused off the
    fused data-parallel path (CPU here)."""
    from rl_b200.models.config import ModelConfig
    from rl_b200.models.transformer import TransformerLM
    from rl_b200.parallel.dist_optimizer import FlatAdamW

    cfg = ModelConfig(name="t", vocab_size=64, hidden_size=32, num_layers=2, num_heads=2, num_kv_heads=1, head_dim=16,
                      ffn_hidden_size=64, rope_theta=10000.0, max_position_embeddings=64)
    m = TransformerLM(cfg, device="cpu", dtype=torch.float32, seed=0)
    opt = FlatAdamW(m, lr=1e-3)
    assert opt.setup_overlap(lambda n: None) is False  # not the fused DP path
    seg = opt.segments[0]
    lo, hi = seg.s_lo, seg.s_hi
    opt._ov = {"done": {0, 1}, "mine": {0: [(lo + 64, lo + 128)], 1: [(lo + 256, lo + 320)], 2: [(lo, lo + 8)]}}
    assert opt._overlap_rest(seg) == [(lo, lo + 64), (lo + 128, lo + 256), (lo + 320, hi)]
    opt._ov["done"] = set()
    assert opt._overlap_rest(seg) == [(lo, hi)]


def test_freeze_moe_router_keeps_router_weights():
    """``megatron_cfg.freeze_moe_router``: a training step moves the experts and
    attention but leaves every router weight bit-identical (no gradient, no
    weight decay)."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY_MOE, make_batch

    pcfg = {"max_total_sequence_length": 32, "precision": "float32", "train_global_batch_size": 8,
            "optimizer": {"kwargs": {"lr": 1e-2, "weight_decay": 0.1}},
            "megatron_cfg": {"freeze_moe_router": True},
            "generation": {"temperature": 1.0, "max_new_tokens": 4},
            "sequence_packing": {"train_mb_tokens": 64, "logprob_mb_tokens": 64}}
    w = PolicyWorker(pcfg, model_cfg=TINY_MOE, seed=3)
    before = {n: p.detach().clone() for n, p in w.model._params.items()}
    w.train(make_batch(B=8, S=24), ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}))
    for n, p in w.model._params.items():
        if n.endswith("mlp.gate.weight"):
            assert torch.equal(p, before[n]), n
    moved = [n for n, p in w.model._params.items() if not torch.equal(p, before[n])]
    assert any("experts" in n for n in moved) and any("qkv" in n for n in moved)


def test_expert_bias_load_balancing():
    """``moe_router_enable_expert_bias``: the bias starts at zero, moves against
    each expert's load after every step (overloaded experts down), steers the
    top-k choice, and never enters the gating weights."""
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.models.policy.worker import PolicyWorker
    from tests.dist_cases import TINY_MOE, make_batch

    pcfg = {"max_total_sequence_length": 32, "precision": "float32", "train_global_batch_size": 8,
            "optimizer": {"kwargs": {"lr": 1e-4}},
            "megatron_cfg": {"moe_router_enable_expert_bias": True, "moe_router_bias_update_rate": 0.01},
            "generation": {"temperature": 1.0, "max_new_tokens": 4},
            "sequence_packing": {"train_mb_tokens": 64, "logprob_mb_tokens": 64}}
    w = PolicyWorker(pcfg, model_cfg=TINY_MOE, seed=3)
    m = w.model
    assert all(float(b.abs().sum()) == 0 for b in m.expert_bias.values())
    res = w.train(make_batch(B=8, S=24), ClippedPGLossFn({"reference_policy_kl_penalty": 0.0}))
    assert "moe/max_load_ratio" in res and res["moe/max_load_ratio"] >= 1.0
    b0 = m.expert_bias[0]
    assert float(b0.abs().max()) == pytest.approx(0.01) and float(b0.max()) > 0 > float(b0.min())
    # selection follows the bias, weights do not
    h = torch.randn(16, TINY_MOE.hidden_size)
    with torch.no_grad():
        m.expert_bias[0] = torch.zeros(TINY_MOE.num_experts)
        m.expert_bias[0][3] = 10.0  # expert 3 always chosen
        vals, ids, probs, _ = m.route(0, h)
    assert bool((ids == 3).any(1).all())
    raw = probs.gather(-1, ids)
    torch.testing.assert_close(vals, raw / raw.sum(-1, keepdim=True))
