"""Eagle3 draft head (CPU): greedy speculative rollouts equal plain greedy
rollouts token for token, online training on the policy's own rollouts lowers
the draft loss and raises the acceptance of its proposals."""

from __future__ import annotations

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict


def _worker(draft: bool, seed=3):
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker

    pcfg = {"max_total_sequence_length": 80, "precision": "float32", "train_global_batch_size": 8,
            "generation": {"temperature": 1.0, "max_new_tokens": 24, "speculative": {"num_speculative_tokens": 3},
                           "mcore_generation_config": {"block_size_tokens": 16}}}
    if draft:
        pcfg["draft"] = {"enabled": True, "speculator_type": "eagle3", "lr": 3e-3, "ttt_steps": 2}
    else:
        pcfg["generation"].pop("speculative")
    return PolicyWorker(pcfg, model_cfg=get_model_config("tiny-llama"), seed=seed)


def _prompts(n=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    return BatchedDataDict({"input_ids": torch.randint(0, 512, (n, 20), generator=g),
                            "input_lengths": torch.randint(6, 21, (n,), generator=g)})


def test_eagle3_greedy_speculation_is_exact():
    plain = _worker(False).generate(_prompts(), greedy=True)
    w = _worker(True)
    spec = w.generate(_prompts(), greedy=True)
    assert torch.equal(spec["output_ids"], plain["output_ids"])
    st = w.engine.spec_stats
    assert st["rounds"] > 0 and st["proposed"] > 0


def test_eagle3_online_training_raises_acceptance():
    w = _worker(True)
    data = _prompts(16, seed=1)
    roll = w.generate(data, greedy=True)
    seqs = BatchedDataDict({"input_ids": roll["output_ids"], "input_lengths": roll["unpadded_sequence_lengths"]})

    def acceptance():
        w.engine.spec_stats = {"rounds": 0, "proposed": 0, "emitted": 0}
        w.generate(data, greedy=True)
        s = w.engine.spec_stats
        return (s["emitted"] - s["rounds"]) / max(1, s["proposed"])  # accepted drafts per proposal (approx.)

    before = acceptance()
    losses = [w.train_draft(seqs) for _ in range(40)]
    after = acceptance()
    assert losses[-1] < 0.5 * losses[0], losses[::8]
    assert after > before + 0.1, (before, after)


def test_mtp_head_speculation_is_exact():
    """``speculator_type: mtp``: the head reads only the last layer's features."""
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker

    pcfg = {"max_total_sequence_length": 80, "precision": "float32", "train_global_batch_size": 8,
            "generation": {"temperature": 1.0, "max_new_tokens": 24, "speculative": {"num_speculative_tokens": 2},
                           "mcore_generation_config": {"block_size_tokens": 16}},
            "draft": {"enabled": True, "speculator_type": "mtp"}}
    w = PolicyWorker(pcfg, model_cfg=get_model_config("tiny-llama"), seed=3)
    assert w.draft.aux_layers == (get_model_config("tiny-llama").num_layers - 1,)
    plain = _worker(False).generate(_prompts(), greedy=True)
    assert torch.equal(w.generate(_prompts(), greedy=True)["output_ids"], plain["output_ids"])
