"""Asynchronous GRPO: replay buffer of prompt groups and a background rollout pump.

Reference behaviour (``nemo_rl/algorithms/async_utils/replay_buffer.py:428-1154``,
``trajectory_collector.py:138-1348``):

* every buffered entry is ONE prompt group (the prompt's G samples) tagged with
  the weight version that generated it and the trainer step (target version)
  it is meant for;
* the trainer at weight version ``v`` takes exactly ``num_prompt_groups`` groups
  whose target is ``v`` and whose generation version is within
  ``max_trajectory_age_steps`` of ``v``; if not enough are ready it waits (so no
  group misses the step it was generated for), stale groups are evicted;
* the rollout pump generating with weights ``w`` may fill the targets
  ``w+1 .. w+lead`` (``initial .. initial+lead`` before the first update), where
  ``lead`` is the maximum trajectory age; it idles when all of them are filled.

Here the pump is a host thread of the same SPMD rank (no actor framework):
generation and training share the GPU, so the pump takes ``weights_lock`` around
each rollout and the trainer takes it around the optimizer step + refit
(``in_flight_weight_updates: false``); with in-flight updates on, the pump only
holds the lock while it snapshots the version, and a rollout that spans an
update is tagged with the version it started from.
"""

from __future__ import annotations

import threading
import time
from collections import Counter
from typing import Any, Optional

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["ReplayBuffer", "AsyncTrajectoryCollector", "split_groups"]


class ReplayBuffer:
    """Thread-safe buffer of per-prompt trajectory groups."""

    def __init__(self, max_size: int):
        if max_size <= 0:
            raise ValueError(f"max_size must be positive, got {max_size}")
        self.max_size = int(max_size)
        self._groups: list[Any] = []
        self._gen_versions: list[int] = []
        self._targets: list[int] = []
        self.last_consumed_target = -1
        self._lock = threading.Lock()

    # ---------------------------------------------------------------- writes
    def add(self, group: Any, weight_version: int, target_weight_version: int) -> str:
        """Append one group; returns ``"full"`` (nothing added) or ``"success"``."""
        with self._lock:
            if len(self._groups) >= self.max_size:
                return "full"
            self._groups.append(group)
            self._gen_versions.append(int(weight_version))
            self._targets.append(int(target_weight_version))
            return "success"

    def _drop(self, idx) -> None:
        for i in sorted(set(idx), reverse=True):
            del self._groups[i], self._gen_versions[i], self._targets[i]

    def sample(self, num_prompt_groups: int, current_weight_version: int,
               max_age_steps: int) -> Optional[dict]:
        """Take the groups meant for step ``current_weight_version`` (FIFO), or
        ``None`` when fewer than ``num_prompt_groups`` of them are ready."""
        with self._lock:
            oldest = max(0, current_weight_version - max_age_steps)
            stale = [i for i, v in enumerate(self._gen_versions) if v < oldest]
            if stale:
                self._drop(stale)
            ready = [i for i, (v, t) in enumerate(zip(self._gen_versions, self._targets))
                     if oldest <= v <= current_weight_version and t == current_weight_version]
            if len(ready) < num_prompt_groups:
                return None
            take = ready[:num_prompt_groups]
            groups = [self._groups[i] for i in take]
            versions = [self._gen_versions[i] for i in take]
            self._drop(take)
            self.last_consumed_target = max(self.last_consumed_target, current_weight_version)
            return {"trajectories": groups,
                    "avg_trajectory_age": current_weight_version - sum(versions) / len(versions),
                    "generation_versions": dict(Counter(versions))}

    def clear(self) -> None:
        with self._lock:
            self._groups.clear()
            self._gen_versions.clear()
            self._targets.clear()

    # ----------------------------------------------------------------- reads
    def size(self) -> int:
        with self._lock:
            return len(self._groups)

    def count_for_target(self, target: int) -> int:
        with self._lock:
            return sum(1 for t in self._targets if t == target)

    def trajectories_needed(self, target: int, num_prompt_groups: int) -> int:
        return max(0, num_prompt_groups - self.count_for_target(target))

    def has_complete_batch(self, target: int, num_prompt_groups: int) -> bool:
        return self.trajectories_needed(target, num_prompt_groups) == 0

    def existing_targets(self) -> set[int]:
        with self._lock:
            return set(self._targets)

    # ------------------------------------------------------------ checkpoint
    def state_dict(self) -> dict:
        with self._lock:
            return {"groups": list(self._groups), "gen_versions": list(self._gen_versions),
                    "targets": list(self._targets), "last_consumed_target": self.last_consumed_target,
                    "max_size": self.max_size}

    def load_state_dict(self, sd: dict, drop_incomplete_targets: Optional[int] = None) -> None:
        """Restore; with ``drop_incomplete_targets=n`` targets holding fewer than
        ``n`` groups are discarded (their prompts are not replayed)."""
        with self._lock:
            self._groups = list(sd["groups"])
            self._gen_versions = [int(v) for v in sd["gen_versions"]]
            self._targets = [int(t) for t in sd["targets"]]
            self.last_consumed_target = int(sd.get("last_consumed_target", -1))
            if drop_incomplete_targets:
                cnt = Counter(self._targets)
                bad = [i for i, t in enumerate(self._targets) if cnt[t] < drop_incomplete_targets]
                self._drop(bad)


def split_groups(rollout: BatchedDataDict, group_size: int) -> list[BatchedDataDict]:
    """Cut a rollout batch whose rows are prompt-major (G consecutive samples per
    prompt) into per-prompt groups."""
    n = len(rollout["message_log"])
    if n % group_size:
        raise ValueError(f"{n} rows is not a multiple of the group size {group_size}")
    return [rollout.select_indices(list(range(i, i + group_size))) for i in range(0, n, group_size)]


class AsyncTrajectoryCollector:
    """Background rollout pump feeding a ``ReplayBuffer``.

    ``rollout_fn(batch) -> (rollout, metrics)`` runs the (multi-turn) rollout of
    one dataloader batch of prompts already repeated G times; the collector
    tags each resulting group with (generation version, target step)."""

    def __init__(self, rollout_fn, dataloader, buffer: ReplayBuffer, num_prompt_groups: int, group_size: int,
                 max_trajectory_age_steps: int = 1, initial_weight_version: int = 0,
                 in_flight_weight_updates: bool = False, max_generation_failures: int = 0,
                 ledger=None, restart_groups: Optional[list] = None, max_group_attempts: Optional[int] = None):
        self.rollout_fn = rollout_fn
        self.dataloader = dataloader
        self.buffer = buffer
        self.num_prompt_groups = int(num_prompt_groups)
        self.group_size = int(group_size)
        self.lead = max(1, int(max_trajectory_age_steps))
        self.initial_weight_version = int(initial_weight_version)
        self.weight_version = int(initial_weight_version)
        self.in_flight_weight_updates = bool(in_flight_weight_updates)
        self.max_generation_failures = int(max_generation_failures)
        self.weights_lock = threading.RLock()
        self._cv = threading.Condition()
        self._generating: set[int] = set()
        self._stop = threading.Event()
        self._running = threading.Event()
        self._running.set()
        self._error: Optional[BaseException] = None
        self._failures = 0
        self._thread: Optional[threading.Thread] = None
        self.exhausted = False
        self.stats = {"groups_generated": 0, "rollouts": 0, "idle_s": 0.0, "gen_s": 0.0, "groups_regenerated": 0}
        # rollout recovery: every prompt group is recorded from dataloader to
        # consumption; groups in flight at a restart are served before new prompts
        self.ledger = ledger
        self.retry_queue: list = list(restart_groups or [])
        self.max_group_attempts = max_group_attempts

    # ----------------------------------------------------------- scheduling
    def target_candidates(self, gen_version: int) -> list[int]:
        if gen_version == self.initial_weight_version:
            return list(range(self.initial_weight_version, self.initial_weight_version + self.lead + 1))
        return [gen_version + i for i in range(1, self.lead + 1)]

    def _reserve_target(self, gen_version: int) -> Optional[int]:
        with self._cv:
            for t in self.target_candidates(gen_version):
                if t <= self.buffer.last_consumed_target or t in self._generating:
                    continue
                if self.buffer.trajectories_needed(t, self.num_prompt_groups) <= 0:
                    continue
                self._generating.add(t)
                return t
        return None

    def set_weight_version(self, version: int) -> None:
        with self._cv:
            self.weight_version = int(version)
            self._cv.notify_all()

    def pause(self) -> None:
        self._running.clear()

    def resume(self) -> None:
        self._running.set()
        with self._cv:
            self._cv.notify_all()

    # ------------------------------------------------------------ lifecycle
    def start(self) -> "AsyncTrajectoryCollector":
        self._thread = threading.Thread(target=self._loop, name="rollout-pump", daemon=True)
        self._thread.start()
        return self

    def stop(self, timeout_s: float = 600.0) -> None:
        self._stop.set()
        self.resume()
        if self._thread is not None:
            self._thread.join(timeout=timeout_s)

    def check_health(self) -> None:
        if self._error is not None:
            raise RuntimeError("rollout pump failed") from self._error

    def _wait(self, pred, timeout_s: float = 0.05) -> None:
        with self._cv:
            if not pred():
                self._cv.wait(timeout=timeout_s)

    def _loop(self) -> None:
        try:
            it = iter(self.dataloader)
            batch = None
            while not self._stop.is_set():
                if not self._running.is_set():
                    self._running.wait(0.05)
                    continue
                v = self.weight_version
                target = self._reserve_target(v)
                if target is None:
                    t0 = time.perf_counter()
                    self._wait(lambda: self.weight_version != v or self._stop.is_set())
                    self.stats["idle_s"] += time.perf_counter() - t0
                    continue
                try:
                    if batch is None:
                        batch, group_ids = self._next_prompts(it, target, v)
                        if batch is None:
                            self.exhausted = True
                            with self._cv:
                                self._generating.discard(target)
                            return
                    if self.ledger is not None:
                        for gid in group_ids:
                            self.ledger.mark_dispatched(gid, target)
                        batch["recovery_group_id"] = list(group_ids)
                    t0 = time.perf_counter()
                    if self.in_flight_weight_updates:
                        with self.weights_lock:
                            gen_version = self.weight_version
                        rollout, _ = self.rollout_fn(batch, target)
                    else:
                        with self.weights_lock:
                            gen_version = self.weight_version
                            rollout, _ = self.rollout_fn(batch, target)
                    self.stats["gen_s"] += time.perf_counter() - t0
                    self.stats["rollouts"] += 1
                    for i, g in enumerate(split_groups(rollout, self.group_size)):
                        if self.ledger is not None:  # sealed before the trainer can consume it
                            self.ledger.mark_group_sealed(group_ids[i], g["total_reward"].tolist()
                                                          if "total_reward" in g else None)
                        while self.buffer.add(g, gen_version, target) == "full":
                            if self._stop.is_set():
                                return
                            time.sleep(0.01)
                        self.stats["groups_generated"] += 1
                    batch = None
                except Exception as e:  # a failed rollout: count it, maybe retry the prompts
                    self._failures += 1
                    if self.ledger is not None and batch is not None:
                        for gid in group_ids:  # retried first unless out of attempts
                            if self.ledger.mark_failed(gid, self.max_group_attempts):
                                self.retry_queue.insert(0, self.ledger.get_group(gid))
                    if self._failures > self.max_generation_failures:
                        raise
                    batch = None
                    del e
                finally:
                    with self._cv:
                        self._generating.discard(target)
                        self._cv.notify_all()
        except BaseException as e:  # surfaced to the trainer by check_health()
            self._error = e

    def _next_prompts(self, it, target: int, version: int):
        """(batch, group ids): prompt groups to regenerate first, else the next
        dataloader batch (its rows reserved in the ledger)."""
        if self.ledger is not None and self.retry_queue:
            n = max(1, self.num_prompt_groups)
            take, self.retry_queue = self.retry_queue[:n], self.retry_queue[n:]
            from rl_b200.experience.rollout_recovery import collate_datums

            self.stats["groups_regenerated"] += len(take)
            return collate_datums([g.prompt for g in take]), [g.group_id for g in take]
        try:
            batch = next(it)
        except StopIteration:
            return None, []
        if self.ledger is None:
            return batch, []
        from rl_b200.experience.rollout_recovery import datum_rows

        ids = [self.ledger.reserve_group(row, self.group_size, target, version) for row in datum_rows(batch)]
        return batch, ids

    def efficiency_metrics(self) -> dict[str, float]:
        tot = self.stats["idle_s"] + self.stats["gen_s"]
        return {"rollout_pump_idle_frac": self.stats["idle_s"] / tot if tot > 0 else 0.0,
                "groups_generated": float(self.stats["groups_generated"]),
                "groups_regenerated": float(self.stats["groups_regenerated"])}


def wait_for_groups(buffer: ReplayBuffer, collector: AsyncTrajectoryCollector, n_groups: int, version: int,
                    max_age: int, timeout_s: float = 3600.0) -> dict:
    """Block until the buffer can serve step ``version`` (checking the pump's
    health while waiting)."""
    t0 = time.perf_counter()
    while True:
        s = buffer.sample(n_groups, version, max_age)
        if s is not None:
            s["wait_s"] = time.perf_counter() - t0
            return s
        collector.check_health()
        if collector.exhausted and not collector._generating and buffer.count_for_target(version) < n_groups:
            raise StopIteration("dataloader exhausted")
        if time.perf_counter() - t0 > timeout_s:
            raise TimeoutError(f"no complete batch for step {version} after {timeout_s:.0f}s")
        with collector._cv:
            collector._cv.wait(timeout=0.02)


def groups_to_batch(groups: list) -> BatchedDataDict:
    return BatchedDataDict.from_batches(groups) if len(groups) > 1 else groups[0]


def torch_state(obj: Any) -> Any:
    """Detach tensors of a buffer state for ``torch.save``."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu()
    if isinstance(obj, dict):
        return {k: torch_state(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [torch_state(v) for v in obj]
    return obj
