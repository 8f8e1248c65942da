"""Parity contract with the reference's clipped policy-gradient loss: loss and
gradients of every golden case (PPO token / sequence ratios, force-on-policy,
REINFORCE, dual clip, CISPO, TIS / ICEPOP / seq-mask-TIS, GSPO, on-policy KL
with unfiltered log-probs, VAPO positive NLL) in float64.

Golden values: the reference's ``tests/unit/algorithms/data/clipped_pg_loss_goldens.json``."""

import copy
import json
import os

import pytest
import torch

from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn

G = json.load(open(os.path.join(os.path.dirname(__file__), "data", "clipped_pg_goldens.json")))


@pytest.mark.parametrize("case", G["cases"], ids=[c["name"] for c in G["cases"]])
def test_clipped_pg_golden(case):
    inp = copy.deepcopy(G["base_inputs"])
    inp.update(copy.deepcopy(case["input_overrides"]))

    def t(k):
        return torch.tensor(inp[k], dtype=torch.int64 if k == "input_ids" else torch.float64)

    lp = t("next_token_logprobs").requires_grad_(True)
    data = {k: t(k) for k in ("input_ids", "token_mask", "sample_mask", "advantages", "prev_logprobs",
                              "generation_logprobs", "reference_policy_logprobs", "rewards")}
    wrt, names = [lp], ["next_token_logprobs"]
    if "curr_logprobs_unfiltered" in inp:
        data["curr_logprobs_unfiltered"] = t("curr_logprobs_unfiltered").requires_grad_(True)
        wrt.append(data["curr_logprobs_unfiltered"])
        names.append("curr_logprobs_unfiltered")
    fn = ClippedPGLossFn(dict(case["config"]))
    gseqs = data["sample_mask"].sum()
    gtoks = (data["token_mask"][:, 1:] * data["sample_mask"].unsqueeze(-1)).sum()
    loss, _ = fn(lp, data, gseqs, gtoks)
    grads = torch.autograd.grad(loss, wrt)
    torch.testing.assert_close(loss.detach(), torch.tensor(case["loss"], dtype=torch.float64), rtol=1e-10, atol=1e-10)
    for n, g in zip(names, grads):
        torch.testing.assert_close(g, torch.tensor(case["gradients"][n], dtype=torch.float64), rtol=1e-9, atol=1e-10)
