"""Flow-GRPO on a toy conditional flow model: the SDE transition log-probs are
the exact Gaussian densities of the sampled steps, and GRPO training moves the
generated points toward the prompt-specific targets."""

import copy
import math

import torch

from rl_b200.research.flow_grpo import (ToyFlowModel, flow_grpo_train, group_advantages, sample_trajectory,
                                        sde_mean_std, transition_logprobs)

TARGETS = torch.tensor([[2.0, 2.0], [-2.0, 2.0], [2.0, -2.0], [-2.0, -2.0]])


def reward(x, cond):
    return -((x - TARGETS[cond]) ** 2).sum(-1)


def test_transition_logprobs_and_window():
    torch.manual_seed(0)
    m = ToyFlowModel()
    cond = torch.tensor([0, 1, 2])
    tr = sample_trajectory(m, cond, steps=6, sde_window=(2, 4), generator=torch.Generator().manual_seed(1))
    assert tr.sde_steps == [2, 3] and tr.logps.shape == (3, 2)
    lp, kl = transition_logprobs(m, tr, ref_model=copy.deepcopy(m))
    torch.testing.assert_close(lp, tr.logps, atol=1e-5, rtol=0)
    assert torch.allclose(kl, torch.zeros_like(kl))
    # the recorded density is N(mu, s^2) of the sampled point
    i = tr.sde_steps[0]
    mu, s, _ = sde_mean_std(m, tr.xs[i], tr.ts[i], tr.ts[i + 1], cond, 0.7)
    z = (tr.xs[i + 1] - mu) / s
    ref = (-0.5 * z ** 2 - math.log(s) - 0.5 * math.log(2 * math.pi)).sum(-1)
    torch.testing.assert_close(tr.logps[:, 0], ref, atol=1e-5, rtol=0)
    adv = group_advantages(torch.tensor([1.0, 2.0, 3.0, 4.0]), 2, leave_one_out=True)
    assert adv[0] < 0 < adv[1] and adv[2] < 0 < adv[3]


def test_flow_grpo_improves_reward():
    torch.manual_seed(0)
    m = ToyFlowModel()
    ref = copy.deepcopy(m)
    before = reward(sample_trajectory(m, torch.arange(4).repeat(64), 10,
                                      generator=torch.Generator().manual_seed(5)).xs[-1],
                    torch.arange(4).repeat(64)).mean()
    log = flow_grpo_train(m, reward, 4, {"max_num_steps": 60, "prompts_per_step": 4, "num_generations_per_prompt": 8,
                                         "lr": 3e-3, "steps": 10, "inner_epochs": 2, "beta": 0.01,
                                         "sde_window_size": 6}, ref_model=ref, seed=0)
    after = reward(sample_trajectory(m, torch.arange(4).repeat(64), 10,
                                     generator=torch.Generator().manual_seed(5)).xs[-1],
                   torch.arange(4).repeat(64)).mean()
    assert after > before + 1.0, (float(before), float(after))
    assert all(math.isfinite(r["policy_loss"]) for r in log)
