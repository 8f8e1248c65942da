"""Rollout engine prefill: identical prompts prefilled once (their KV blocks
copied to the group's other rows) and prefill split into passes of at most
``max_tokens`` tokens give the same greedy rollouts and log-probs as one plain
prefill (CPU)."""

from __future__ import annotations

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict


def _worker(mg: dict, device="cpu"):
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.parallel.state import single_process_state

    pcfg = {"max_total_sequence_length": 96, "precision": "float32" if device == "cpu" else "bfloat16",
            "train_global_batch_size": 12,
            "generation": {"temperature": 1.0, "max_new_tokens": 12,
                           "mcore_generation_config": {"block_size_tokens": 16, **mg}}}
    return PolicyWorker(pcfg, model_cfg=get_model_config("tiny-llama"),
                        pstate=single_process_state(torch.device(device)), seed=3)


def _batch(G=3):
    g = torch.Generator().manual_seed(0)
    lens = torch.tensor([5, 23, 40, 17])
    ids = torch.randint(0, 512, (4, 40), generator=g)
    return BatchedDataDict({"input_ids": ids.repeat_interleave(G, 0), "input_lengths": lens.repeat_interleave(G)})


def test_dedup_and_chunked_prefill_match_plain_prefill():
    data = _batch()
    ref_w = _worker({"enable_prefix_caching": False, "enable_chunked_prefill": False})
    ref = ref_w.generate(data, greedy=True)
    assert ref_w.engine.stats_last_prefill == {"prompts": 12, "prefilled": 12, "passes": 1, "tokens": 255}
    w = _worker({"enable_prefix_caching": True, "enable_chunked_prefill": True, "max_tokens": 30})
    out = w.generate(data, greedy=True)
    st = w.engine.stats_last_prefill
    assert st["prefilled"] == 4 and st["tokens"] == 85 and st["passes"] == 3, st  # [5, 23] [40] [17]
    assert torch.equal(out["output_ids"], ref["output_ids"])
    torch.testing.assert_close(out["logprobs"], ref["logprobs"], atol=1e-5, rtol=0)
    # sampled rollouts of one group still differ from each other after the shared prefill
    s = w.generate(data)
    ids = s["output_ids"]
    assert not (torch.equal(ids[0], ids[1]) and torch.equal(ids[1], ids[2]))
