"""Forest training: training rows from the captured model calls of one
logical rollout (context compaction, retries, branches).

An agent harness may rewrite its own history between model calls (compact
it, retry a rejected answer, branch).  Every model call is captured with a
link to the call whose exact tokens it continues:

* a **root** (``parent_id is None``) holds its whole input ``input_ids`` and
  the generated ``output_ids`` (a first call, or a call whose context was
  rewritten);
* a **continuation** holds only its new input tokens (the observation after
  the parent's answer) and its output; the parent's tokens are the prefix.

Given the calls a rollout actually *kept* (``select_calls``), the rows are
the paths from each root to each selected endpoint (a selected call with no
selected child): the concatenated inputs and outputs along the path, with the
generated spans as loss tokens.  A call shared by several paths is context
in every one of them but carries loss only in the first (endpoints in
capture order), so every kept generated token is trained exactly once.  All
rows of a rollout share its single reward: advantages are computed once per
logical rollout (``owner``) within its prompt group and broadcast to the
rows (``owner_advantages``).

Selection policies (``token_capture.selection_policy``): ``returned_history``
keeps the calls the harness returned (every kept continuation's parent must
be kept too: a gap is an error, not a silent cut); ``all_captured`` keeps
every call except failed / unknown leaves that are not the scored call, and
incomplete leaves whose finish reason is not ``length``.  A kept call that
failed, or a failed parent, masks the whole rollout.

Reference: ``docs/guides/context-compaction.md`` (forest reconstruction,
once-only loss ownership, selection policies) and the logical-owner
advantage stage (``nemo_rl/algorithms/single_controller_utils/logical_advantage.py:32``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

__all__ = ["CapturedCall", "ForestRow", "select_calls", "reconstruct_rows", "rollout_rows", "owner_advantages",
           "fanout"]


@dataclass
class CapturedCall:
    call_id: str
    parent_id: Optional[str]
    input_ids: list[int]
    output_ids: list[int]
    output_logprobs: Optional[list[float]] = None
    status: str = "completed"        # completed | incomplete | failed | unknown
    finish_reason: str = "stop"      # stop | length | ...


@dataclass
class ForestRow:
    token_ids: torch.Tensor
    token_loss_mask: torch.Tensor
    generation_logprobs: torch.Tensor
    call_ids: list[str] = field(default_factory=list)


def _by_id(calls: Sequence[CapturedCall]) -> dict[str, CapturedCall]:
    out = {}
    for c in calls:
        if c.call_id in out:
            raise ValueError(f"duplicate call id {c.call_id!r}")
        out[c.call_id] = c
    for c in calls:
        if c.parent_id is not None and c.parent_id not in out:
            raise ValueError(f"call {c.call_id!r} continues unknown call {c.parent_id!r}")
    return out


def select_calls(calls: Sequence[CapturedCall], policy: str = "returned_history",
                 returned_ids: Optional[Sequence[str]] = None, terminal_id: Optional[str] = None) -> list[str]:
    """Ids of the calls that train, in capture order."""
    byid = _by_id(calls)
    if policy == "returned_history":
        if returned_ids is None:
            raise ValueError("returned_history selection needs the harness's returned call ids")
        keep = set(returned_ids)
        unknown = keep - set(byid)
        if unknown:
            raise ValueError(f"returned history names calls that were never captured: {sorted(unknown)}")
        for cid in keep:
            p = byid[cid].parent_id
            if p is not None and p not in keep:
                raise ValueError(f"kept call {cid!r} continues {p!r}, which the returned history omits")
    elif policy == "all_captured":
        if terminal_id is None or terminal_id not in byid:
            raise ValueError("all_captured selection needs the scored terminal call id")
        has_child = {c.parent_id for c in calls if c.parent_id is not None}
        keep = set()
        for c in calls:
            leaf = c.call_id not in has_child
            dropped = leaf and c.call_id != terminal_id and (
                c.status in ("failed", "unknown") or (c.status == "incomplete" and c.finish_reason != "length"))
            if not dropped:
                keep.add(c.call_id)
    else:
        raise ValueError(f"unknown selection policy {policy!r} (returned_history, all_captured)")
    if terminal_id is not None and terminal_id not in keep:
        raise ValueError(f"the scored call {terminal_id!r} is not among the kept calls")
    return [c.call_id for c in calls if c.call_id in keep]


def rollout_valid(calls: Sequence[CapturedCall], selected: Sequence[str]) -> bool:
    """A kept call that failed (or has an unknown outcome) invalidates the rollout."""
    byid = _by_id(calls)
    return all(byid[c].status not in ("failed", "unknown") for c in selected)


def reconstruct_rows(calls: Sequence[CapturedCall], selected: Sequence[str]) -> list[ForestRow]:
    byid = _by_id(calls)
    sel = [c for c in (x.call_id for x in calls) if c in set(selected)]
    sel_set = set(sel)
    parents_of_selected = {byid[c].parent_id for c in sel if byid[c].parent_id is not None}
    endpoints = [c for c in sel if c not in parents_of_selected]
    owned: set[str] = set()
    rows = []
    for end in endpoints:
        path = []
        cur: Optional[str] = end
        while cur is not None:
            if cur not in sel_set:
                raise ValueError(f"path to {end!r} crosses unselected call {cur!r}")
            path.append(cur)
            cur = byid[cur].parent_id
        path.reverse()
        ids, mask, lps = [], [], []
        for cid in path:
            c = byid[cid]
            train = cid not in owned
            owned.add(cid)
            ids += list(c.input_ids) + list(c.output_ids)
            mask += [0] * len(c.input_ids) + [1 if train else 0] * len(c.output_ids)
            out_lp = list(c.output_logprobs) if c.output_logprobs is not None else [0.0] * len(c.output_ids)
            if len(out_lp) != len(c.output_ids):
                raise ValueError(f"call {cid!r}: {len(out_lp)} logprobs for {len(c.output_ids)} output tokens")
            lps += [0.0] * len(c.input_ids) + out_lp
        rows.append(ForestRow(torch.tensor(ids, dtype=torch.long), torch.tensor(mask, dtype=torch.float32),
                              torch.tensor(lps, dtype=torch.float32), path))
    return rows


def rollout_rows(calls: Sequence[CapturedCall], policy: str = "returned_history",
                 returned_ids: Optional[Sequence[str]] = None, terminal_id: Optional[str] = None
                 ) -> tuple[list[ForestRow], bool]:
    """Rows of one logical rollout and whether it may train (``False``: mask
    every row of it, e.g. a kept call failed)."""
    sel = select_calls(calls, policy, returned_ids, terminal_id)
    rows = reconstruct_rows(calls, sel)
    return rows, rollout_valid(calls, sel)


def owner_advantages(estimator, group_ids: torch.Tensor, rewards: torch.Tensor,
                     valid: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One advantage per logical rollout from the run's advantage estimator
    (GRPO, Reinforce++, ...): each owner is one "sequence" of one token, so
    baselines and normalisation see every rollout once, however many rows it
    was split into.  Invalid owners do not vote (``valid_mask``)."""
    n = rewards.numel()
    adv = estimator.compute_advantage(group_ids.view(-1, 1), rewards.float(), torch.ones(n, 1),
                                      valid_mask=None if valid is None else valid.float())
    if isinstance(adv, tuple):
        adv = adv[0]
    adv = adv.view(n, -1)[:, 0]
    return adv if valid is None else adv * valid.float()


def fanout(values: torch.Tensor, row_owner: torch.Tensor) -> torch.Tensor:
    """One value per owner broadcast to its rows; ownerless padding (-1) gets 0."""
    return values[row_owner.clamp_min(0)] * (row_owner >= 0)
