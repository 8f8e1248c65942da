"""NVFP4 rollout weights (CPU): real NVFP4 storage (packed e2m1 codes, e4m3
block scales, fp32 tensor scale) round-trips to the fake quantiser's values;
the rollout samples from the NVFP4-weight model while the trained weights stay
bf16 / fp32 untouched."""

from __future__ import annotations

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict
from rl_b200.models.quantization import QuantSpec, dequant_nvfp4, fake_quant, quant_nvfp4


def test_nvfp4_storage_round_trip():
    torch.manual_seed(0)
    for shape in [(64, 128), (33, 40), (8, 16)]:
        w = torch.randn(*shape) * 0.05
        t = quant_nvfp4(w)
        assert t.codes.dtype == torch.uint8 and t.codes.shape == (shape[0], -(-shape[1] // 16) * 8)
        assert t.block_scales.dtype == torch.float8_e4m3fn
        torch.testing.assert_close(dequant_nvfp4(t), fake_quant(w, QuantSpec("nvfp4", (1, 16))), atol=0, rtol=0)
    w = torch.randn(256, 256)
    assert quant_nvfp4(w).nbytes < 0.3 * w.numel() * 2  # ~4.5 bits per weight vs 16


def test_rollout_uses_nvfp4_weights():
    from rl_b200.models.config import get_model_config
    from rl_b200.models.policy.worker import PolicyWorker
    from rl_b200.weight_sync.colocated import NVFP4RolloutSynchronizer

    mcfg = get_model_config("tiny-llama")

    def worker(prec):
        pcfg = {"max_total_sequence_length": 64, "precision": "float32", "train_global_batch_size": 4,
                "generation": {"temperature": 1.0, "max_new_tokens": 12, "vllm_cfg": {"precision": prec},
                               "mcore_generation_config": {"block_size_tokens": 16}}}
        return PolicyWorker(pcfg, model_cfg=mcfg, seed=5)

    g = torch.Generator().manual_seed(0)
    data = BatchedDataDict({"input_ids": torch.randint(0, mcfg.vocab_size, (4, 16), generator=g),
                            "input_lengths": torch.tensor([16, 9, 12, 5])})
    w = worker("nvfp4")
    before = w.model.flat_param.detach().clone()
    w.refit()
    out = w.generate(data, greedy=True)
    assert torch.equal(w.model.flat_param, before)  # training weights untouched
    assert w.weight_sync.stats["nvfp4_bytes"] > 0
    # the same model with its linear weights fake-quantised by hand generates the same tokens
    ref = worker("bfloat16")
    with torch.no_grad():
        ref.model.flat_param.copy_(before)
        for sp, p in ref.model.named_flat_params():
            if NVFP4RolloutSynchronizer.quantized(sp.name):
                p.copy_(fake_quant(p.view(-1, p.shape[-1]), QuantSpec("nvfp4", (1, 16))).view(p.shape))
    ref.refit()
    assert torch.equal(out["output_ids"], ref.generate(data, greedy=True)["output_ids"])
