"""Flow-GRPO: online RL for flow-matching (rectified-flow) generators.

A deterministic ODE sampler has no likelihood, so the rollout integrates the
marginal-preserving SDE of the rectified flow ``x_t = (1 - t) x_0 + t x_1``
(``t`` runs from 1 = noise to 0 = data, velocity ``v = x_1 - x_0``):

    dx = [v(x, t) + sigma_t^2 / (2 t) * (x + (1 - t) v(x, t))] dt + sigma_t dW,
    sigma_t = a * sqrt(t / (1 - t))

(Liu et al., "Flow-GRPO", 2025).  With Euler-Maruyama each denoising step is
a Gaussian ``x_next ~ N(mu_theta(x_t), s^2 I)``, ``s = sigma_t sqrt(|dt|)``, so
its log-probability is closed-form and differentiable in the model.  Training
then follows GRPO: G samples per prompt, group-relative advantages of a
terminal reward, per-step ratios ``exp(log p_new - log p_old)`` in the clipped
objective, optional KL to the reference model (for equal variances the Gaussian
KL is ``|mu_theta - mu_ref|^2 / (2 s^2)``).  ``sde_window`` makes only a slice of
the steps stochastic (the "Fast" variant): the loss recomputes only those.

``ToyFlowModel`` (a small conditional MLP velocity field over points) keeps the
algorithm testable without an image model; any module with
``forward(x, t, cond) -> v`` plugs in.

Reference: ``research/flow_grpo/`` of the reference (README "How It Works",
SDE step ``flow_grpo/algorithms/sde.py``, loss ``flow_grpo/algorithms/loss/flow_grpo.py``,
loop ``flow_grpo/algorithms/flow_grpo.py``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn as nn

__all__ = ["ToyFlowModel", "sde_mean_std", "sample_trajectory", "transition_logprobs", "flow_grpo_loss",
           "group_advantages", "flow_grpo_train", "Trajectory"]


class ToyFlowModel(nn.Module):
    def __init__(self, dim: int = 2, n_cond: int = 4, hidden: int = 64):
        super().__init__()
        self.emb = nn.Embedding(n_cond, hidden)
        self.net = nn.Sequential(nn.Linear(dim + 1 + hidden, hidden), nn.SiLU(), nn.Linear(hidden, hidden), nn.SiLU(),
                                 nn.Linear(hidden, dim))

    def forward(self, x: torch.Tensor, t: torch.Tensor, cond: torch.Tensor) -> torch.Tensor:
        return self.net(torch.cat([x, t.expand(x.shape[0], 1), self.emb(cond)], -1))


def sde_mean_std(model, x: torch.Tensor, t: float, t_next: float, cond: torch.Tensor, a: float):
    """Mean and std of the Euler-Maruyama step t -> t_next (t_next < t)."""
    tt = torch.full((1, 1), t, dtype=x.dtype, device=x.device)
    v = model(x, tt, cond)
    dt = t_next - t
    tc = min(max(t, 1e-4), 1 - 1e-4)
    sigma = a * math.sqrt(tc / (1 - tc))
    drift = v + (sigma ** 2) / (2 * tc) * (x + (1 - tc) * v)
    return x + drift * dt, sigma * math.sqrt(abs(dt)), v


@dataclass
class Trajectory:
    xs: list          # x at every step boundary [N, dim] (len steps + 1)
    logps: torch.Tensor  # [N, n_sde] log-probs of the stochastic steps (rollout policy)
    sde_steps: list   # indices of the stochastic steps
    cond: torch.Tensor
    ts: list


def _gauss_logp(x: torch.Tensor, mu: torch.Tensor, s: float) -> torch.Tensor:
    d = x.shape[-1]
    return -((x - mu) ** 2).sum(-1) / (2 * s * s) - d * math.log(s) - 0.5 * d * math.log(2 * math.pi)


@torch.no_grad()
def sample_trajectory(model, cond: torch.Tensor, steps: int = 10, a: float = 0.7, dim: int = 2,
                      sde_window: Optional[tuple] = None, generator: Optional[torch.Generator] = None) -> Trajectory:
    """Sample ``len(cond)`` trajectories from noise (t = 1) to data (t = 0):
    steps inside ``sde_window`` ([first, end) step indices; default all) are
    stochastic, the others follow the ODE."""
    N = cond.shape[0]
    ts = [1.0 - i / steps for i in range(steps + 1)]
    ts[0] = 1.0 - 1e-3  # the SDE coefficient is singular at t = 1
    w0, w1 = sde_window if sde_window is not None else (0, steps)
    x = torch.randn(N, dim, generator=generator)
    xs, lps, sde_steps = [x], [], []
    for i in range(steps):
        t, tn = ts[i], ts[i + 1]
        mu, s, v = sde_mean_std(model, x, t, tn, cond, a)
        if w0 <= i < w1 and tn > 0:
            x = mu + s * torch.randn(x.shape, generator=generator)
            lps.append(_gauss_logp(x, mu, s))
            sde_steps.append(i)
        else:
            x = x + v * (tn - t)  # ODE step
        xs.append(x)
    logps = torch.stack(lps, 1) if lps else torch.zeros(N, 0)
    return Trajectory(xs, logps, sde_steps, cond, ts)


def transition_logprobs(model, traj: Trajectory, a: float = 0.7, ref_model=None):
    """Log-probs of the recorded stochastic steps under ``model`` (with grad),
    and the per-step Gaussian KL to ``ref_model`` when given."""
    lps, kls = [], []
    for i in traj.sde_steps:
        t, tn = traj.ts[i], traj.ts[i + 1]
        mu, s, _ = sde_mean_std(model, traj.xs[i], t, tn, traj.cond, a)
        lps.append(_gauss_logp(traj.xs[i + 1], mu, s))
        if ref_model is not None:
            with torch.no_grad():
                mu_r, _, _ = sde_mean_std(ref_model, traj.xs[i], t, tn, traj.cond, a)
            kls.append(((mu - mu_r) ** 2).sum(-1) / (2 * s * s))
    lp = torch.stack(lps, 1)
    kl = torch.stack(kls, 1) if kls else None
    return lp, kl


def group_advantages(rewards: torch.Tensor, group: int, leave_one_out: bool = False, global_std: bool = True,
                     eps: float = 1e-4) -> torch.Tensor:
    r = rewards.view(-1, group)
    if leave_one_out and group > 1:
        base = (r.sum(1, keepdim=True) - r) / (group - 1)
    else:
        base = r.mean(1, keepdim=True)
    std = rewards.std() if global_std else r.std(1, keepdim=True)
    return ((r - base) / (std + eps)).reshape(-1)


def flow_grpo_loss(new_lp: torch.Tensor, old_lp: torch.Tensor, adv: torch.Tensor, clip: float = 0.2,
                   kl: Optional[torch.Tensor] = None, beta: float = 0.0, adv_clip: float = 5.0):
    """Clipped objective over every stochastic step of every sample."""
    adv = adv.clamp(-adv_clip, adv_clip).unsqueeze(1)
    ratio = torch.exp(new_lp - old_lp)
    pg = torch.maximum(-adv * ratio, -adv * ratio.clamp(1 - clip, 1 + clip)).mean()
    loss = pg + (beta * kl.mean() if (kl is not None and beta > 0) else 0.0)
    return loss, {"policy_loss": float(pg.detach()), "clip_frac": float(((ratio - 1).abs() > clip).float().mean()),
                  "kl": float(kl.detach().mean()) if kl is not None else 0.0}


def flow_grpo_train(model, reward_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor], n_prompts: int,
                    cfg: dict, ref_model=None, seed: int = 0) -> list[dict]:
    """``reward_fn(samples [N, dim], cond [N]) -> [N]``.  cfg keys: steps,
    num_generations_per_prompt, prompts_per_step, lr, clip, beta, noise_level,
    sde_window_size, inner_epochs, max_num_steps, leave_one_out, global_std."""
    G = int(cfg.get("num_generations_per_prompt", 8))
    P = int(cfg.get("prompts_per_step", 4))
    steps = int(cfg.get("steps", 10))
    a = float(cfg.get("noise_level", 0.7))
    win = cfg.get("sde_window_size")
    opt = torch.optim.AdamW(model.parameters(), lr=float(cfg.get("lr", 1e-3)), weight_decay=0.0)
    g = torch.Generator().manual_seed(seed)
    log = []
    for step in range(int(cfg.get("max_num_steps", 10))):
        cond = torch.randint(0, n_prompts, (P,), generator=g).repeat_interleave(G)
        window = None
        if win:
            w0 = int(torch.randint(0, max(1, steps - int(win) + 1), (1,), generator=g))
            window = (w0, w0 + int(win))
        traj = sample_trajectory(model, cond, steps, a, sde_window=window, generator=g)
        rewards = reward_fn(traj.xs[-1], cond)
        adv = group_advantages(rewards, G, bool(cfg.get("leave_one_out", False)), bool(cfg.get("global_std", True)))
        for _ in range(int(cfg.get("inner_epochs", 1))):
            new_lp, kl = transition_logprobs(model, traj, a, ref_model)
            loss, m = flow_grpo_loss(new_lp, traj.logps, adv, float(cfg.get("clip", 0.2)), kl,
                                     float(cfg.get("beta", 0.0)))
            opt.zero_grad(set_to_none=True)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), float(cfg.get("max_grad_norm", 1.0)))
            opt.step()
        m.update(reward_mean=float(rewards.mean()), step=step)
        log.append(m)
    return log
