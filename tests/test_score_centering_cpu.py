"""Score centering: with the sampler equal to the policy and the whole
vocabulary as the head, the correction's gradient is exactly the negated
sampler-expected score (it cancels the REINFORCE drift), untruncated IS needs
no correction, and the loss adds A * term."""

import torch

from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
from rl_b200.algorithms.loss.score_centering import score_centering_term


def test_term_is_the_expected_score():
    torch.manual_seed(0)
    logits = torch.randn(2, 3, 5, requires_grad=True)
    lp = torch.log_softmax(logits, -1)
    mask = torch.ones(2, 3)
    # sampler = policy over the full vocabulary (k = V): rho = 0/0 -> head mass 1, alpha = 0
    term, head = score_centering_term(lp, lp.detach(), "off", None, mask)
    torch.testing.assert_close(head, torch.ones(2, 3))
    g = torch.autograd.grad(term.sum(), logits)[0]
    # sum_v p_v grad log p_v = 0: the expected score of the full distribution vanishes
    torch.testing.assert_close(g, torch.zeros_like(g), atol=1e-6, rtol=0)
    # a sampler different from the policy: coefficient q - rho p on the head
    q = torch.log_softmax(torch.randn(2, 3, 5), -1)
    term2, _ = score_centering_term(lp[..., :3], q[..., :3], "off", None, mask)
    p, qq = lp.detach().exp()[..., :3], q.exp()[..., :3]
    rho = (1 - qq.sum(-1)) / (1 - p.sum(-1))
    torch.testing.assert_close(term2, ((qq - rho.unsqueeze(-1) * p) * lp[..., :3].detach()).sum(-1))
    z, _ = score_centering_term(lp[..., :3], q[..., :3], "is", None, mask)
    torch.testing.assert_close(z, torch.zeros_like(z))


def test_clipped_pg_with_score_centering():
    torch.manual_seed(1)
    B, S, k = 2, 5, 4
    lp_full = torch.log_softmax(torch.randn(B, S - 1, 8), -1)
    ids = torch.randint(0, 8, (B, S - 1, k))
    plk = lp_full.gather(-1, ids).requires_grad_(True)
    data = {"token_mask": torch.ones(B, S), "sample_mask": torch.ones(B), "advantages": torch.randn(B, S),
            "prev_logprobs": torch.zeros(B, S), "generation_logprobs": torch.zeros(B, S),
            "sampler_topk_logprobs": torch.cat([torch.zeros(B, 1, k), lp_full.gather(-1, ids) - 0.1], 1)}
    data["token_mask"][:, 0] = 0
    curr = lp_full[..., 0].clone().requires_grad_(True)
    gs, gt = data["sample_mask"].sum(), data["token_mask"][:, 1:].sum()
    base, _ = ClippedPGLossFn({})(curr, data, gs, gt)
    fn = ClippedPGLossFn({"score_centering": True})
    loss, m = fn(curr, data, gs, gt, policy_logprobs_at_sampler_topk=plk)
    term, _ = score_centering_term(plk, data["sampler_topk_logprobs"][:, 1:], "off", None,
                                   data["token_mask"][:, 1:])
    torch.testing.assert_close(loss, base + (data["advantages"][:, 1:] * term).sum() / gt)
    assert "score_centering_head_mass" in m


def test_engine_records_sampler_topk_and_grpo_trains_with_centering():
    """The rollout records the sampler's top-k of each generated token's
    distribution (the sampled token's log-prob is among them when it is in the
    top-k), and a GRPO run with score centering trains."""
    import os

    from examples.run_grpo import main
    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from tests.test_core_cpu import _tiny_policy

    w = _tiny_policy(seed=7, generation={"temperature": 1.0, "max_new_tokens": 6})
    w.engine.record_sampler_topk = 4
    g = torch.Generator().manual_seed(0)
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (3, 8), generator=g),
                            "input_lengths": torch.tensor([8, 5, 7])})
    out = w.generate(data)
    ids, lps = out["sampler_topk_token_ids"], out["sampler_topk_logprobs"]
    assert ids.shape[:2] == out["output_ids"].shape and ids.shape[-1] == 4
    for b in range(3):
        L, n = int(data["input_lengths"][b]), int(out["generation_lengths"][b])
        for j in range(L, L + n):
            assert (lps[b, j, :-1] >= lps[b, j, 1:]).all()  # sorted top-k
            tok = int(out["output_ids"][b, j])
            hit = (ids[b, j] == tok).nonzero()
            if hit.numel():
                assert abs(float(lps[b, j, hit[0, 0]]) - float(out["logprobs"][b, j])) < 1e-4
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    state = main(["--config", os.path.join(root, "examples", "configs", "grpo_tiny_cpu.yaml"),
                  "logger.log_dir=/tmp/rlb_test_logs_sc", "logger.stdout=false", "grpo.max_num_steps=1",
                  "++loss_fn.score_centering=true", "++loss_fn.score_centering_topk=4"])
    assert state["current_step"] == 1
