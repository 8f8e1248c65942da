"""Liveness state machine for the generation shards, a load-aware shard selector
and a restart supervisor.

Reference: ``ShardState`` / ``GenerationFleetHealth`` / ``HealthyShardSelector``
(``nemo_rl/models/generation/fleet_health.py:43-610``) and ``EngineSupervisor``
(``nemo_rl/models/generation/engine_supervisor.py:55``).  The six states and the
rule that matters most are the reference's: a shard that died never becomes
HEALTHY by answering probes again; a restarted engine holds stale weights, so
it goes RESTARTING -> STALE and only a completed refit to the trainer's current
weight version makes it HEALTHY.

Everything here is host bookkeeping (no I/O): probes, restarts and refits are
performed by the caller and reported in, so every transition is testable on CPU.
"""

from __future__ import annotations

import enum
import itertools
import threading
import time
from dataclasses import dataclass
from typing import Callable, Optional

__all__ = ["ShardState", "ShardHealth", "FleetHealthPolicy", "GenerationFleetHealth", "GenerationFleetExhausted",
           "HealthyShardSelector", "EngineSupervisor"]


class ShardState(str, enum.Enum):
    HEALTHY = "healthy"        # serving, weights current
    SUSPECT = "suspect"        # failing probes, still served (a blip must not drain a shard)
    DEAD = "dead"              # quarantined, no replacement yet
    RESTARTING = "restarting"  # replacement coming up
    STALE = "stale"            # alive but holding old weights: not served until refit
    RETIRED = "retired"        # terminal


SERVING = frozenset({ShardState.HEALTHY, ShardState.SUSPECT})
# cannot take part in a collective (refit) - SUSPECT / STALE can, which is how STALE recovers
ABSENT = frozenset({ShardState.DEAD, ShardState.RESTARTING, ShardState.RETIRED})


@dataclass
class ShardHealth:
    idx: int
    state: ShardState = ShardState.HEALTHY
    probe_failures: int = 0
    probe_successes: int = 0
    reported_failures: int = 0
    restart_attempts: int = 0
    weight_version: int = 0
    last_ok_at: float = 0.0
    last_error: str = ""

    @property
    def serving(self) -> bool:
        return self.state in SERVING


class GenerationFleetExhausted(RuntimeError):
    pass


@dataclass
class FleetHealthPolicy:
    unhealthy_threshold: int = 3
    healthy_threshold: int = 2
    max_restart_attempts_per_shard: int = 5
    min_healthy_shards: int = 1

    def __post_init__(self):
        if min(self.unhealthy_threshold, self.healthy_threshold) < 1:
            raise ValueError("thresholds must be >= 1")
        if self.max_restart_attempts_per_shard < 0 or self.min_healthy_shards < 0:
            raise ValueError("limits must be >= 0")


class GenerationFleetHealth:
    def __init__(self, num_shards: int, policy: Optional[FleetHealthPolicy] = None,
                 on_transition: Optional[Callable[[int, ShardState, ShardState], None]] = None):
        self.policy = policy or FleetHealthPolicy()
        self.shards = [ShardHealth(i) for i in range(int(num_shards))]
        self.on_transition = on_transition
        self.membership_epoch = 0
        self.trainer_version = 0
        self._lock = threading.RLock()
        self.transitions: list[tuple[int, str, str]] = []

    # ----------------------------------------------------------------- views
    def state_of(self, i: int) -> ShardState:
        return self.shards[i].state

    def serving_shards(self) -> list[int]:
        with self._lock:
            return [s.idx for s in self.shards if s.serving]

    def absent_shards(self) -> list[int]:
        with self._lock:
            return [s.idx for s in self.shards if s.state in ABSENT]

    def counts(self) -> dict[str, int]:
        with self._lock:
            out = {st.value: 0 for st in ShardState}
            for s in self.shards:
                out[s.state.value] += 1
            return out

    def as_metrics(self) -> dict[str, float]:
        c = self.counts()
        m = {f"fleet/{k}": float(v) for k, v in c.items()}
        m["fleet/membership_epoch"] = float(self.membership_epoch)
        return m

    # ----------------------------------------------------------- transitions
    def _set(self, s: ShardHealth, new: ShardState) -> None:
        old = s.state
        if old == new:
            return
        was_absent = old in ABSENT
        s.state = new
        self.transitions.append((s.idx, old.value, new.value))
        if was_absent != (new in ABSENT):
            self.membership_epoch += 1
        if self.on_transition is not None:
            self.on_transition(s.idx, old, new)

    def record_probe(self, i: int, ok: bool, error: str = "") -> None:
        with self._lock:
            s = self.shards[i]
            if s.state in ABSENT:
                return
            if ok:
                s.probe_failures = 0
                s.probe_successes += 1
                s.last_ok_at = time.monotonic()
                if s.state == ShardState.SUSPECT and s.probe_successes >= self.policy.healthy_threshold \
                        and s.reported_failures == 0:
                    self._set(s, ShardState.HEALTHY)
                return
            s.probe_successes = 0
            s.probe_failures += 1
            s.last_error = error
            if s.state == ShardState.HEALTHY:
                self._set(s, ShardState.SUSPECT)
            if s.probe_failures >= self.policy.unhealthy_threshold:
                self._set(s, ShardState.DEAD)

    def report_failure(self, i: int, error: BaseException | str) -> None:
        """A real request failed.  Counted apart from probes: a wedged engine can
        keep answering probes, so only ``report_success`` or a refit clears it."""
        with self._lock:
            s = self.shards[i]
            if s.state in ABSENT:
                return
            s.reported_failures += 1
            s.last_error = str(error)
            if s.state == ShardState.HEALTHY:
                self._set(s, ShardState.SUSPECT)
            if s.reported_failures >= self.policy.unhealthy_threshold:
                self._set(s, ShardState.DEAD)

    def report_success(self, i: int) -> None:
        with self._lock:
            s = self.shards[i]
            s.reported_failures = 0
            s.last_ok_at = time.monotonic()

    def record_death(self, i: int, error: str = "") -> None:
        with self._lock:
            s = self.shards[i]
            if s.state != ShardState.RETIRED:
                s.last_error = error
                self._set(s, ShardState.DEAD)

    def mark_restarting(self, i: int) -> bool:
        """DEAD -> RESTARTING (False, and RETIRED, once restarts are exhausted)."""
        with self._lock:
            s = self.shards[i]
            if s.state != ShardState.DEAD:
                return False
            if s.restart_attempts >= self.policy.max_restart_attempts_per_shard:
                self._set(s, ShardState.RETIRED)
                return False
            s.restart_attempts += 1
            self._set(s, ShardState.RESTARTING)
            return True

    def mark_loaded(self, i: int) -> None:
        """The replacement answers: STALE until a refit brings it to the trainer's weights."""
        with self._lock:
            s = self.shards[i]
            if s.state == ShardState.RESTARTING:
                s.probe_failures = s.probe_successes = s.reported_failures = 0
                self._set(s, ShardState.STALE)

    def mark_restart_failed(self, i: int, error: str = "") -> None:
        with self._lock:
            s = self.shards[i]
            if s.state == ShardState.RESTARTING:
                s.last_error = error
                self._set(s, ShardState.RETIRED if s.restart_attempts >= self.policy.max_restart_attempts_per_shard
                          else ShardState.DEAD)

    def report_refit(self, i: int, weight_version: int) -> None:
        """A completed refit: STALE -> HEALTHY when the shard now holds the
        trainer's current version; reported failures are cleared."""
        with self._lock:
            s = self.shards[i]
            if s.state in ABSENT:
                return
            s.weight_version = int(weight_version)
            s.reported_failures = 0
            if s.state == ShardState.STALE and s.weight_version >= self.trainer_version:
                self._set(s, ShardState.HEALTHY)

    def set_trainer_version(self, v: int) -> None:
        with self._lock:
            self.trainer_version = int(v)

    def retire(self, i: int, reason: str = "") -> None:
        with self._lock:
            self.shards[i].last_error = reason
            self._set(self.shards[i], ShardState.RETIRED)

    def raise_if_exhausted(self) -> None:
        n = len(self.serving_shards())
        if n < self.policy.min_healthy_shards:
            raise GenerationFleetExhausted(f"{n} serving shards < min_healthy_shards={self.policy.min_healthy_shards}: "
                                           f"{self.counts()}")


class HealthyShardSelector:
    """Pick the serving shard with the fewest requests in flight (round-robin
    among ties); callers ``acquire`` / ``release`` around each request."""

    def __init__(self, fleet: GenerationFleetHealth):
        self.fleet = fleet
        self._inflight = [0] * len(fleet.shards)
        self._rr = itertools.count()
        self._lock = threading.Lock()

    def next_shard(self) -> int:
        serving = self.fleet.serving_shards()
        if not serving:
            raise GenerationFleetExhausted("no serving generation shard")
        with self._lock:
            lo = min(self._inflight[i] for i in serving)
            cands = [i for i in serving if self._inflight[i] == lo]
            return cands[next(self._rr) % len(cands)]

    def acquire(self, i: int) -> None:
        with self._lock:
            self._inflight[i] += 1

    def release(self, i: int) -> None:
        with self._lock:
            self._inflight[i] = max(0, self._inflight[i] - 1)

    def inflight(self, i: int) -> int:
        return self._inflight[i]


class EngineSupervisor:
    """Restarts DEAD shards through ``restart_fn(shard) -> None`` (raising on
    failure) on background threads; ``tick()`` is called from the training loop."""

    def __init__(self, fleet: GenerationFleetHealth, restart_fn: Callable[[int], None], max_concurrent: int = 1):
        self.fleet = fleet
        self.restart_fn = restart_fn
        self.max_concurrent = int(max_concurrent)
        self._threads: dict[int, threading.Thread] = {}
        self.restarts_ok = 0
        self.restarts_failed = 0

    def tick(self) -> None:
        for i, t in list(self._threads.items()):
            if not t.is_alive():
                del self._threads[i]
        for s in self.fleet.shards:
            if len(self._threads) >= self.max_concurrent:
                break
            if s.state == ShardState.DEAD and s.idx not in self._threads and self.fleet.mark_restarting(s.idx):
                t = threading.Thread(target=self._run, args=(s.idx,), daemon=True, name=f"restart-{s.idx}")
                self._threads[s.idx] = t
                t.start()

    def _run(self, i: int) -> None:
        try:
            self.restart_fn(i)
        except Exception as e:  # noqa: BLE001 - a failed restart is state, not a crash
            self.restarts_failed += 1
            self.fleet.mark_restart_failed(i, repr(e))
            return
        self.restarts_ok += 1
        self.fleet.mark_loaded(i)

    def join(self, timeout_s: float = 30.0) -> None:
        for t in list(self._threads.values()):
            t.join(timeout_s)

    def as_metrics(self) -> dict[str, float]:
        return {"fleet/restarts_ok": float(self.restarts_ok), "fleet/restarts_failed": float(self.restarts_failed),
                "fleet/restarts_in_flight": float(len(self._threads))}
