"""Rollout recovery ledger: the controller's record of every prompt group between
leaving the dataloader and being consumed by a training step, so a restart
regenerates exactly the groups that were in flight.

Reference: ``nemo_rl/experience/rollout_recovery.py`` (``RolloutRecoveryLedger``
``:611``, checkpoint file ``rollout_recovery.pt``).  Same purpose and lifecycle
(reserve -> dispatch -> per-sibling seal -> group seal -> consumed, with
versioned ``state_dict`` written at each checkpoint and strict schema checks on
load); the reference's NeMo-Gym episode and TransferQueue staging bookkeeping
is not modelled (neither exists here).

Why it is needed: the dataloader's checkpointed position is already past every
prompt the rollout pump has taken.  Prompts whose groups were still being
generated, or whose trajectories sat in a replay buffer that is not restored,
would otherwise be skipped silently after a restart.  The ledger keeps each
group's prompt (the dataset row: message log with token ids, environment info)
until a training step consumes it; ``prepare_for_restart`` returns the groups to
generate again, and the rollout pump serves them before asking the dataloader
for new prompts.
"""

from __future__ import annotations

import copy
import functools
import threading
import uuid
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Iterable, Optional

import torch

__all__ = ["GroupStatus", "AttemptStatus", "PromptRef", "AttemptRecord", "SiblingRecord", "GroupRecord",
           "RolloutRecoveryLedger", "ROLLOUT_RECOVERY_SCHEMA_VERSION", "ROLLOUT_RECOVERY_STATE_FILENAME",
           "datum_rows", "collate_datums"]

ROLLOUT_RECOVERY_SCHEMA_VERSION = 1
ROLLOUT_RECOVERY_STATE_FILENAME = "rollout_recovery.pt"


class GroupStatus(str, Enum):
    RESERVED = "reserved"      # taken from the dataloader, not yet generating
    DISPATCHED = "dispatched"  # a rollout of its siblings is running
    SEALED = "sealed"          # every sibling finished; trajectories in the replay buffer
    ABANDONED = "abandoned"    # given up (failure budget exhausted); not regenerated


class AttemptStatus(str, Enum):
    RUNNING = "running"
    SEALED = "sealed"
    FAILED = "failed"
    ABANDONED = "abandoned"    # in flight when the process stopped


@dataclass
class PromptRef:
    sample_id: int
    task_name: str


@dataclass
class AttemptRecord:
    attempt_uuid: str
    status: AttemptStatus = AttemptStatus.RUNNING
    reward: Optional[float] = None


@dataclass
class SiblingRecord:
    generation_index: int
    attempts: list[AttemptRecord] = field(default_factory=list)

    @property
    def sealed(self) -> bool:
        return bool(self.attempts) and self.attempts[-1].status == AttemptStatus.SEALED


@dataclass
class GroupRecord:
    group_id: str
    prompt_ref: PromptRef
    prompt: dict                     # the dataset row (DatumSpec) this group generates from
    expected_generations: int
    target_step: int
    start_weight_version: int
    status: GroupStatus = GroupStatus.RESERVED
    siblings: list[SiblingRecord] = field(default_factory=list)

    def unsealed_indices(self) -> list[int]:
        return [s.generation_index for s in self.siblings if not s.sealed]


_GROUP_FIELDS = {"group_id", "prompt_ref", "prompt", "expected_generations", "target_step", "start_weight_version",
                 "status", "siblings"}
_SIBLING_FIELDS = {"generation_index", "attempts"}
_ATTEMPT_FIELDS = {"attempt_uuid", "status", "reward"}


def _check_fields(d: dict, allowed: set, what: str) -> None:
    extra = set(d) - allowed
    missing = allowed - set(d)
    if extra or missing:
        raise ValueError(f"{what}: unknown fields {sorted(extra)} / missing fields {sorted(missing)}")


def _locked(fn):
    @functools.wraps(fn)
    def wrapper(self, *a, **kw):
        with self._lock:
            return fn(self, *a, **kw)
    return wrapper


class RolloutRecoveryLedger:
    """Lineage of in-flight prompt groups (control data only: the prompt row and
    per-attempt status; generated tokens stay in the replay buffer).  Safe to use
    from the rollout-pump thread and the trainer thread at once."""

    def __init__(self):
        self._groups: dict[str, GroupRecord] = {}
        self._lock = threading.RLock()

    # --------------------------------------------------------------- queries
    def __len__(self) -> int:
        return len(self._groups)

    def __contains__(self, group_id: object) -> bool:
        return group_id in self._groups

    def get_group(self, group_id: str) -> GroupRecord:
        if group_id not in self._groups:
            raise KeyError(f"unknown prompt group {group_id!r}")
        return self._groups[group_id]

    @property
    def groups(self) -> list[GroupRecord]:
        return list(self._groups.values())

    @_locked
    def counts(self) -> dict[str, int]:
        out = {s.value: 0 for s in GroupStatus}
        for g in self._groups.values():
            out[g.status.value] += 1
        return out

    # ------------------------------------------------------------- lifecycle
    @_locked
    def reserve_group(self, prompt: dict, expected_generations: int, target_step: int, weight_version: int,
                      group_id: Optional[str] = None) -> str:
        """Record a prompt taken for generation; returns its group id."""
        gid = group_id or uuid.uuid4().hex
        if gid in self._groups:
            raise ValueError(f"prompt group {gid!r} already reserved")
        ref = PromptRef(int(prompt.get("idx", -1)), str(prompt.get("task_name", "default")))
        self._groups[gid] = GroupRecord(gid, ref, prompt, int(expected_generations), int(target_step),
                                        int(weight_version),
                                        siblings=[SiblingRecord(i) for i in range(int(expected_generations))])
        return gid

    @_locked
    def mark_dispatched(self, group_id: str, target_step: Optional[int] = None) -> None:
        """A rollout of the group's unsealed siblings starts (one new attempt each)."""
        g = self.get_group(group_id)
        if g.status not in (GroupStatus.RESERVED, GroupStatus.DISPATCHED):
            raise ValueError(f"group {group_id!r} is {g.status.value}; only reserved groups dispatch")
        if target_step is not None:
            g.target_step = int(target_step)
        for s in g.siblings:
            if not s.sealed:
                s.attempts.append(AttemptRecord(uuid.uuid4().hex))
        g.status = GroupStatus.DISPATCHED

    @_locked
    def mark_sibling_sealed(self, group_id: str, generation_index: int, reward: Optional[float] = None) -> None:
        g = self.get_group(group_id)
        s = g.siblings[generation_index]
        if not s.attempts or s.attempts[-1].status != AttemptStatus.RUNNING:
            raise ValueError(f"group {group_id!r} sibling {generation_index} has no running attempt")
        s.attempts[-1].status = AttemptStatus.SEALED
        s.attempts[-1].reward = None if reward is None else float(reward)

    @_locked
    def mark_group_sealed(self, group_id: str, rewards: Optional[Iterable[float]] = None) -> None:
        """All siblings finished and the group's trajectories entered the buffer."""
        g = self.get_group(group_id)
        rewards = list(rewards) if rewards is not None else [None] * len(g.siblings)
        for s, r in zip(g.siblings, rewards):
            if not s.sealed:
                self.mark_sibling_sealed(group_id, s.generation_index, r)
        g.status = GroupStatus.SEALED

    @_locked
    def mark_failed(self, group_id: str, max_attempts: Optional[int] = None) -> bool:
        """The running attempt failed; the group returns to reserved (retried)
        unless a sibling reached ``max_attempts``, then it is abandoned.
        Returns whether it will be retried."""
        g = self.get_group(group_id)
        worst = 0
        for s in g.siblings:
            if s.attempts and s.attempts[-1].status == AttemptStatus.RUNNING:
                s.attempts[-1].status = AttemptStatus.FAILED
            worst = max(worst, len(s.attempts))
        if max_attempts is not None and worst >= max_attempts:
            g.status = GroupStatus.ABANDONED
            return False
        g.status = GroupStatus.RESERVED
        return True

    @_locked
    def mark_consumed(self, group_ids: Iterable[str]) -> None:
        """A training step used these groups: they leave the ledger."""
        for gid in group_ids:
            g = self.get_group(gid)
            if g.status != GroupStatus.SEALED:
                raise ValueError(f"group {gid!r} consumed while {g.status.value}")
            del self._groups[gid]

    @_locked
    def discard(self, group_ids: Iterable[str]) -> None:
        """Groups dropped on purpose (e.g. stale trajectories evicted): forget them."""
        for gid in group_ids:
            self._groups.pop(gid, None)

    @_locked
    def prune_sealed(self, live_ids: Iterable[str]) -> int:
        """Forget sealed groups whose trajectories are no longer in the replay buffer
        (evicted as too old); returns how many were dropped."""
        live = set(live_ids)
        dead = [gid for gid, g in self._groups.items() if g.status == GroupStatus.SEALED and gid not in live]
        for gid in dead:
            del self._groups[gid]
        return len(dead)

    # --------------------------------------------------------------- restart
    @_locked
    def prepare_for_restart(self, buffer_group_ids: Optional[Iterable[str]] = None) -> list[GroupRecord]:
        """Groups to generate again after a restart, in reservation order: every
        reserved or dispatched group (its running attempts are abandoned) and
        every sealed group whose trajectories are not in the restored replay
        buffer (``buffer_group_ids``: the ledger ids the restored buffer holds;
        None = no buffer was restored).  The returned groups are RESERVED again."""
        live = set(buffer_group_ids) if buffer_group_ids is not None else set()
        redo = []
        for g in self._groups.values():
            if g.status == GroupStatus.ABANDONED:
                continue
            if g.status == GroupStatus.SEALED and g.group_id in live:
                continue
            for s in g.siblings:
                if s.attempts and s.attempts[-1].status == AttemptStatus.RUNNING:
                    s.attempts[-1].status = AttemptStatus.ABANDONED
                if g.status == GroupStatus.SEALED:  # trajectories lost with the buffer
                    s.attempts.append(AttemptRecord(uuid.uuid4().hex, AttemptStatus.ABANDONED))
            g.status = GroupStatus.RESERVED
            redo.append(g)
        return redo

    @_locked
    def assert_checkpoint_safe(self) -> None:
        """No attempt may be mid-flight in a checkpoint (the pump is paused)."""
        for g in self._groups.values():
            if g.status == GroupStatus.DISPATCHED:
                raise RuntimeError(f"checkpoint while prompt group {g.group_id!r} is generating")

    # ------------------------------------------------------------ state dict
    @_locked
    def state_dict(self) -> dict[str, Any]:
        groups = []
        for g in self._groups.values():
            groups.append({
                "group_id": g.group_id, "prompt_ref": {"sample_id": g.prompt_ref.sample_id,
                                                       "task_name": g.prompt_ref.task_name},
                "prompt": copy.copy(g.prompt), "expected_generations": g.expected_generations,
                "target_step": g.target_step, "start_weight_version": g.start_weight_version,
                "status": g.status.value,
                "siblings": [{"generation_index": s.generation_index,
                              "attempts": [{"attempt_uuid": a.attempt_uuid, "status": a.status.value,
                                            "reward": a.reward} for a in s.attempts]} for s in g.siblings]})
        return {"schema_version": ROLLOUT_RECOVERY_SCHEMA_VERSION, "groups": groups}

    @classmethod
    def from_state_dict(cls, state: dict[str, Any]) -> "RolloutRecoveryLedger":
        _check_fields(state, {"schema_version", "groups"}, "rollout recovery state")
        if state["schema_version"] != ROLLOUT_RECOVERY_SCHEMA_VERSION:
            raise ValueError(f"unsupported rollout recovery schema {state['schema_version']}")
        led = cls()
        for raw in state["groups"]:
            _check_fields(raw, _GROUP_FIELDS, "prompt group")
            sibs = []
            for rs in raw["siblings"]:
                _check_fields(rs, _SIBLING_FIELDS, "sibling")
                atts = []
                for ra in rs["attempts"]:
                    _check_fields(ra, _ATTEMPT_FIELDS, "attempt")
                    atts.append(AttemptRecord(ra["attempt_uuid"], AttemptStatus(ra["status"]), ra["reward"]))
                sibs.append(SiblingRecord(int(rs["generation_index"]), atts))
            pr = raw["prompt_ref"]
            g = GroupRecord(raw["group_id"], PromptRef(int(pr["sample_id"]), str(pr["task_name"])), raw["prompt"],
                            int(raw["expected_generations"]), int(raw["target_step"]),
                            int(raw["start_weight_version"]), GroupStatus(raw["status"]), sibs)
            if g.group_id in led._groups:
                raise ValueError(f"duplicate prompt group {g.group_id!r}")
            led._groups[g.group_id] = g
        return led

    def save(self, path: str) -> None:
        torch.save(self.state_dict(), path)

    @classmethod
    def load(cls, path: str) -> "RolloutRecoveryLedger":
        return cls.from_state_dict(torch.load(path, map_location="cpu", weights_only=False))


_ROW_KEYS = ("message_log", "extra_env_info", "task_name", "stop_strings")


def datum_rows(batch) -> list[dict]:
    """The dataset rows of a collated prompt batch (inverse of ``rl_collate_fn``)."""
    n = len(batch["message_log"])
    rows = []
    for i in range(n):
        r = {k: batch[k][i] for k in _ROW_KEYS if k in batch}
        r["length"] = int(batch["length"][i]) if "length" in batch else 0
        r["loss_multiplier"] = float(batch["loss_multiplier"][i]) if "loss_multiplier" in batch else 1.0
        r["idx"] = int(batch["idx"][i]) if "idx" in batch else i
        rows.append(r)
    return rows


def collate_datums(rows: list[dict]):
    from rl_b200.data.datasets import rl_collate_fn

    return rl_collate_fn(rows)
