"""Muon (``megatron_cfg.optimizer.optimizer: dist_muon``): the Newton-Schulz
update against ``torch.optim.Muon`` (same algorithm), the tensor-parallel
modes against the full-matrix result, and GRPO training steps through the
policy worker at TP=1 / TP=2 / DP=2 (gloo)."""

import math

import pytest
import torch

from rl_b200.distributed.launch import spawn_ranks
from rl_b200.parallel.muon import MuonConfig, muon_scale, newton_schulz
from tests.dist_cases import case_train_step

MUON = {"optimizer": "dist_muon", "lr": 2e-3, "weight_decay": 0.01, "muon_momentum": 0.9, "muon_nesterov": False,
        "muon_scale_mode": "spectral", "muon_extra_scale_factor": 0.2, "muon_fp32_matmul_prec": "highest",
        "muon_num_ns_steps": 5, "muon_tp_mode": "distributed", "muon_split_qkv": True}


def test_newton_schulz_orthogonalizes():
    g = torch.Generator().manual_seed(0)
    for shape in [(48, 32), (32, 80), (3, 40, 24)]:
        u = torch.randn(*shape, generator=g)
        o = newton_schulz(u, 5)
        s = torch.linalg.svdvals(o)
        assert s.min() > 0.3 and s.max() < 1.3, (shape, s.min(), s.max())


@pytest.mark.parametrize("mode,torch_fn,nesterov", [("spectral", "match_rms_adamw", False),
                                                     ("shape_scaling", "original", True)])
def test_matches_torch_muon(mode, torch_fn, nesterov):
    """Same momentum, NS5, decoupled decay and scale as ``torch.optim.Muon``
    (which runs NS in bf16: compared at bf16 tolerance over three steps)."""
    from rl_b200.parallel.muon import orthogonalize

    g = torch.Generator().manual_seed(1)
    w0 = torch.randn(64, 40, generator=g)
    grads = [torch.randn(64, 40, generator=g) for _ in range(3)]
    lr, wd, mu = 0.02, 0.1, 0.95
    p = torch.nn.Parameter(w0.clone())
    opt = torch.optim.Muon([p], lr=lr, weight_decay=wd, momentum=mu, nesterov=nesterov, adjust_lr_fn=torch_fn)
    cfg = MuonConfig(momentum=mu, nesterov=nesterov, scale_mode=mode, fp32_matmul_prec="highest",
                     extra_scale_factor=0.2 if mode == "spectral" else 1.0)
    w, buf = w0.clone(), torch.zeros_like(w0)
    for gr in grads:
        p.grad = gr.clone()
        opt.step()
        buf.lerp_(gr, 1 - mu)
        upd = gr.lerp(buf, mu) if nesterov else buf
        o, (a, b) = orthogonalize(upd, None, cfg)
        w = w * (1 - lr * wd) - lr * muon_scale(a, b, mode) * cfg.extra_scale_factor * o
    step = (w - w0).abs().max()
    assert (p.detach() - w).abs().max() < 3e-2 * step, ((p.detach() - w).abs().max(), step)


def _tp_case(rank, mode):
    import torch.distributed as dist

    from rl_b200.parallel.muon import orthogonalize
    from rl_b200.parallel.state import init_distributed

    ps = init_distributed(tp=2, backend="gloo")
    g = torch.Generator().manual_seed(5)
    full = torch.randn(2, 40, 24, generator=g)  # batched (experts-like) and 2-D cases below
    cfg = MuonConfig(tp_mode=mode, fp32_matmul_prec="highest")
    out = {}
    for name, x, dim in [("rows", full[0], -2), ("cols", full[1], -1), ("batched_rows", full, -2)]:
        n = x.shape[dim] // 2
        local = x.narrow(dim, rank * n, n)
        o, shape = orthogonalize(local, dim, cfg, ps.tp_group)
        parts = [torch.empty_like(o) for _ in range(2)]
        dist.all_gather(parts, o.contiguous(), group=ps.tp_group)
        out[name] = (torch.cat(parts, dim), shape)
    return out


@pytest.mark.parametrize("mode", ["distributed", "duplicated"])
def test_tp_modes_equal_full_matrix(mode):
    outs = spawn_ranks(_tp_case, 2, mode)
    g = torch.Generator().manual_seed(5)
    full = torch.randn(2, 40, 24, generator=g)
    ref = {"rows": newton_schulz(full[0]), "cols": newton_schulz(full[1]), "batched_rows": newton_schulz(full)}
    for name, r in ref.items():
        got, shape = outs[0][name]
        assert shape == tuple(r.shape[-2:])
        assert (got - r).abs().max() < 1e-4, (mode, name, (got - r).abs().max())


def test_config_validation():
    assert MuonConfig.from_megatron({"optimizer": "adam"}) is None
    with pytest.raises(ValueError, match="muon_tp_mode"):
        MuonConfig.from_megatron({"optimizer": "dist_muon", "muon_tp_mode": "sharded"})
    with pytest.raises(ValueError, match="muon_scale_mode"):
        MuonConfig.from_megatron({"optimizer": "muon", "muon_scale_mode": "rms"})


def test_worker_trains_with_muon_tp_and_dp_match_single():
    single = spawn_ranks(case_train_step, 1, 1, 1, False, False, 1, 1, MUON)[0]
    adam = spawn_ranks(case_train_step, 1, 1, 1, False, False)[0]
    assert math.isfinite(single["loss"]) and not torch.allclose(single["lp"], adam["lp"])
    tp2 = spawn_ranks(case_train_step, 2, 2, 1, False, False, 1, 1, MUON)
    dp2 = spawn_ranks(case_train_step, 2, 1, 1, False, False, 1, 1, MUON)
    for outs in (tp2, dp2):
        for o in outs:
            assert (o["lp"] - single["lp"]).abs().max() < 2e-4, (o["lp"] - single["lp"]).abs().max()
