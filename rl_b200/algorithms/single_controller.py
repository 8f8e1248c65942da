"""SingleController: an asyncio orchestrator for asynchronous GRPO.

Reference: ``nemo_rl/algorithms/single_controller.py:15-39`` (a rollout pump, a
train pump and a stall watchdog coordinating workers; samples move through the
data plane, the controller moves metadata) and the option groups of
``nemo_rl/algorithms/single_controller_utils/config.py`` kept here by name:
``rollout_failure`` (``:119``: per-prompt infra / data attempt budgets, backoff,
skipped-prompt budget, ``min_step_batch_fraction``, ``on_dropped_prompt``),
``stall_watchdog`` (``:464``: ``interval_s``, ``stall_timeout_s``,
``stall_action``), ``max_inflight_prompts`` / ``max_buffered_rollouts`` (``:528-530``).

One controller runs per rank (SPMD; no separate CPU actor).  On a rank:

* the rollout pump takes prompt groups (retries first, once their backoff has
  passed, then new dataloader rows), generates them in a worker thread with the
  current weights, and puts every finished group into the data plane under
  partition ``rollouts``; ``max_inflight_prompts`` bounds one generation call and
  ``max_buffered_rollouts`` stops the pump while that many groups wait;
* the train pump waits for ``num_prompts_per_step / dp`` groups no older than
  ``max_trajectory_age_steps`` versions (older ones are evicted and their prompts
  regenerated), reads them out of the plane, and runs advantages, log-prob passes
  and the split train API (``begin_train_step`` / ``train_microbatch`` /
  ``finish_train_step``) in a worker thread; the update and the refit hold the
  weights lock, so no rollout reads a half-written model;
* the watchdog checks every ``interval_s`` that some pump finished a unit of work
  within ``stall_timeout_s`` and that no worker-thread call has run longer than
  that; ``stall_action: warn`` logs and counts, ``abort`` ends ``run`` with
  ``StallError``.

A failed generation call charges one attempt to each of its prompt groups, as an
``infra`` failure (any exception) or a ``data`` failure (``RolloutDataError``,
``ValueError``); a group past its budget is dropped and counted as skipped, and
more than ``max_skipped_prompts`` skipped prompts ends the run.  With dropped
prompts a step may train on fewer groups (``on_dropped_prompt: shrink``) down to
``min_step_batch_fraction`` of the batch, or wait for replacements from the
dataloader (``replace``).  Under data parallelism every rank takes the count of
groups that all ranks hold (a MIN all-reduce per poll, in lockstep), so the
training collectives stay matched.
"""

from __future__ import annotations

import asyncio
import logging
import math
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch

log = logging.getLogger(__name__)

__all__ = ["SingleController", "RolloutFailurePolicy", "WatchdogConfig", "StallError", "RolloutDataError",
           "single_controller_train"]


class StallError(RuntimeError):
    """Raised by ``SingleController.run`` when the watchdog aborts a stalled run."""


class RolloutDataError(ValueError):
    """A generation failure caused by the prompt itself (charged to the data budget)."""


@dataclass
class RolloutFailurePolicy:
    max_infra_attempts_per_prompt: int = 5
    max_data_attempts_per_prompt: int = 2
    backoff_base_s: float = 1.0
    max_backoff_s: float = 30.0
    max_skipped_prompts: int = 0
    min_step_batch_fraction: float = 0.9
    on_dropped_prompt: str = "shrink"

    @classmethod
    def from_config(cls, cfg: Optional[dict]) -> "RolloutFailurePolicy":
        cfg = dict(cfg or {})
        known = {k: cfg[k] for k in cls.__dataclass_fields__ if k in cfg}
        p = cls(**known)
        if p.on_dropped_prompt not in ("shrink", "replace"):
            raise ValueError(f"rollout_failure.on_dropped_prompt must be shrink or replace, got {p.on_dropped_prompt!r}")
        if not 0.0 < p.min_step_batch_fraction <= 1.0:
            raise ValueError("rollout_failure.min_step_batch_fraction must be in (0, 1]")
        return p

    @staticmethod
    def classify(exc: BaseException) -> str:
        return "data" if isinstance(exc, (RolloutDataError, ValueError)) else "infra"

    def budget(self, kind: str) -> int:
        return self.max_data_attempts_per_prompt if kind == "data" else self.max_infra_attempts_per_prompt

    def backoff_s(self, attempt: int) -> float:
        """Delay before attempt ``attempt + 1`` (exponential, capped)."""
        return min(self.max_backoff_s, self.backoff_base_s * (2.0 ** max(0, attempt - 1)))


@dataclass
class WatchdogConfig:
    interval_s: float = 30.0
    stall_timeout_s: float = 600.0
    stall_action: str = "warn"

    @classmethod
    def from_config(cls, cfg: Optional[dict]) -> "WatchdogConfig":
        cfg = dict(cfg or {})
        w = cls(**{k: cfg[k] for k in cls.__dataclass_fields__ if k in cfg})
        if w.stall_action not in ("warn", "abort"):
            raise ValueError(f"stall_watchdog.stall_action must be warn or abort, got {w.stall_action!r}")
        return w


@dataclass
class _PromptWork:
    """One prompt group on its way through the rollout pump."""
    gid: str
    prompt: Any                 # one datum (dict of per-row values) of the dataloader batch
    attempts: dict = field(default_factory=lambda: {"infra": 0, "data": 0})
    not_before: float = 0.0     # monotonic time the next attempt may start


class SingleController:
    """Rollout pump + train pump + watchdog over one rank's policy.

    ``generate_fn(batch, version) -> rollout`` generates a collated batch of
    prompts (each row already repeated ``group_size`` times) and returns the
    rollout ``BatchedDataDict`` (``message_log``, ``total_reward``, ...);
    ``train_fn(groups, version) -> metrics`` trains one step on a list of group
    batches.  ``single_controller_train`` wires both to a ``PolicyWorker``."""

    PARTITION = "rollouts"

    def __init__(self, generate_fn: Callable, train_fn: Callable, dataloader, group_size: int,
                 groups_per_step: int, max_steps: int, cfg: Optional[dict] = None, data_plane=None,
                 initial_version: int = 0, max_trajectory_age_steps: int = 1, dp_group=None,
                 weights_lock: Optional[threading.RLock] = None, on_step: Optional[Callable] = None,
                 ledger=None):
        from rl_b200.data_plane.planes import InProcessDataPlane

        cfg = dict(cfg or {})
        self.generate_fn = generate_fn
        self.train_fn = train_fn
        self.dataloader = dataloader
        self.group_size = int(group_size)
        self.groups_per_step = int(groups_per_step)
        self.max_steps = int(max_steps)
        self.failure = RolloutFailurePolicy.from_config(cfg.get("rollout_failure"))
        self.watchdog = WatchdogConfig.from_config(cfg.get("stall_watchdog"))
        self.max_inflight_prompts = max(1, int(cfg.get("max_inflight_prompts", 32)))
        self.max_buffered_rollouts = max(self.groups_per_step, int(cfg.get("max_buffered_rollouts", 64)))
        self.max_age = max(0, int(max_trajectory_age_steps))
        self.plane = data_plane or InProcessDataPlane()
        self.version = int(initial_version)
        self.dp_group = dp_group
        self.weights_lock = weights_lock or threading.RLock()
        self.on_step = on_step
        self.ledger = ledger
        # group key -> (generation version, gid); the payload lives in the plane
        self._ready: dict[str, tuple[int, str]] = {}
        self._queue: list[_PromptWork] = []          # retries and evicted prompts, served first
        self._exhausted = False
        self._dropped_since_step = 0
        self._seq = 0
        self.stats = {"groups_generated": 0, "groups_evicted": 0, "prompts_skipped": 0, "infra_failures": 0,
                      "data_failures": 0, "retries": 0, "stalls": 0, "shrunk_steps": 0, "gen_calls": 0}
        self.history: list[dict] = []
        self._last_progress = time.monotonic()
        self._busy: dict[str, float] = {}            # pump -> start of its running worker-thread call
        self._wake: Optional[asyncio.Event] = None
        self._done = False

    # ------------------------------------------------------------- helpers
    def _progress(self) -> None:
        self._last_progress = time.monotonic()

    def _notify(self) -> None:
        if self._wake is not None:
            self._wake.set()

    async def _wait_wake(self, timeout: float) -> None:
        try:
            await asyncio.wait_for(self._wake.wait(), timeout)
        except asyncio.TimeoutError:
            pass
        self._wake.clear()

    async def _in_thread(self, pump: str, fn, *args):
        self._busy[pump] = time.monotonic()
        try:
            return await asyncio.get_running_loop().run_in_executor(self._pool, fn, *args)
        finally:
            self._busy.pop(pump, None)

    def _new_gid(self) -> str:
        self._seq += 1
        return f"g{self._seq:08d}"

    def _take_prompts(self, it) -> list[_PromptWork]:
        """Up to ``max_inflight_prompts`` groups: due retries first, then new rows."""
        from rl_b200.experience.rollout_recovery import datum_rows

        now = time.monotonic()
        room = min(self.max_inflight_prompts, self.max_buffered_rollouts - len(self._ready))
        due = [w for w in self._queue if w.not_before <= now][:room]
        for w in due:
            self._queue.remove(w)
        out = list(due)
        while len(out) < room and not self._exhausted:
            try:
                batch = next(it)
            except StopIteration:
                self._exhausted = True
                break
            for row in datum_rows(batch):
                gid = self._new_gid()
                if self.ledger is not None:
                    gid = self.ledger.reserve_group(row, self.group_size, self.version, self.version)
                out.append(_PromptWork(gid, row))
        return out

    def _generate(self, work: list[_PromptWork], version: int):
        from rl_b200.algorithms.async_utils import split_groups
        from rl_b200.experience.rollout_recovery import collate_datums

        batch = collate_datums([w.prompt for w in work]).repeat_interleave(self.group_size)
        with self.weights_lock:  # the weights this call generates with stay fixed
            rollout = self.generate_fn(batch, version)
        return split_groups(rollout, self.group_size)

    def _charge(self, work: list[_PromptWork], exc: BaseException) -> None:
        kind = self.failure.classify(exc)
        self.stats[f"{kind}_failures"] += 1
        for w in work:
            w.attempts[kind] += 1
            if self.ledger is not None and w.gid in self.ledger:
                self.ledger.mark_failed(w.gid, None)
            if w.attempts[kind] >= self.failure.budget(kind):
                self.stats["prompts_skipped"] += 1
                self._dropped_since_step += 1
                if self.ledger is not None:
                    self.ledger.discard([w.gid])  # dropped for good: not regenerated after a restart
                log.warning("prompt group %s dropped after %d %s failures: %s", w.gid, w.attempts[kind], kind, exc)
                if self.stats["prompts_skipped"] > self.failure.max_skipped_prompts:
                    raise RuntimeError(f"{self.stats['prompts_skipped']} prompt groups skipped, more than "
                                       f"rollout_failure.max_skipped_prompts={self.failure.max_skipped_prompts}") \
                        from exc
                continue
            w.not_before = time.monotonic() + self.failure.backoff_s(sum(w.attempts.values()))
            self.stats["retries"] += 1
            self._queue.append(w)

    # --------------------------------------------------------------- pumps
    async def _rollout_pump(self) -> None:
        it = iter(self.dataloader)
        while not self._done:
            if len(self._ready) >= self.max_buffered_rollouts:
                await self._wait_wake(0.05)  # back-pressure: the trainer is behind
                self._progress()              # waiting on the trainer is not a stall of this pump
                continue
            work = self._take_prompts(it)
            if not work:
                if self._exhausted and not self._queue:
                    return
                await self._wait_wake(0.02)   # only retries in backoff remain
                continue
            version = self.version
            if self.ledger is not None:
                for w in work:
                    if w.gid in self.ledger:
                        self.ledger.mark_dispatched(w.gid, version)
            self.stats["gen_calls"] += 1
            try:
                groups = await self._in_thread("rollout", self._generate, work, version)
            except Exception as e:  # noqa: BLE001 - every failure is charged to its prompts
                self._charge(work, e)
                self._notify()
                continue
            for w, g in zip(work, groups):
                key = f"{version:08d}-{w.gid}"
                g["recovery_group_id"] = [w.gid] * len(g["message_log"])
                self.plane.put(self.PARTITION, key, g)
                if self.ledger is not None and w.gid in self.ledger:
                    self.ledger.mark_group_sealed(w.gid, g["total_reward"].tolist() if "total_reward" in g else None)
                self._ready[key] = (version, w.gid)
                self.stats["groups_generated"] += 1
            self._progress()
            self._notify()

    def _evict_stale(self) -> None:
        """Groups generated more than ``max_age`` versions before the next step
        leave the plane; their prompts are generated again."""
        for key, (ver, gid) in list(self._ready.items()):
            if ver < self.version - self.max_age:
                g = self.plane.get(self.PARTITION, key, timeout=5.0)
                self.plane.delete(self.PARTITION, key)
                del self._ready[key]
                self.stats["groups_evicted"] += 1
                from rl_b200.experience.rollout_recovery import datum_rows

                row = _first_row(g, datum_rows)
                if self.ledger is not None and gid in self.ledger:
                    self.ledger.discard([gid])
                    gid = self.ledger.reserve_group(row, self.group_size, self.version, self.version)
                self._queue.insert(0, _PromptWork(gid, row))

    def _agreed(self, n: int, finished: bool) -> tuple[int, bool]:
        """Under data parallelism: the smallest group count over the ranks and
        whether any rank can form no further step (one MIN all-reduce)."""
        import torch.distributed as dist

        if self.dp_group is None or dist.get_world_size(self.dp_group) <= 1:
            return n, finished
        t = torch.tensor([n, -int(finished)], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.dp_group)
        return int(t[0]), bool(t[1] < 0)

    def _step_size(self, have: int, producing: bool) -> int:
        """Groups to train on now (0 = keep waiting)."""
        need = self.groups_per_step
        if have >= need:
            return need
        floor = max(1, math.ceil(self.failure.min_step_batch_fraction * need))
        short_by_drops = self._dropped_since_step > 0 and self.failure.on_dropped_prompt == "shrink"
        if have >= floor and (short_by_drops or not producing):
            return have
        return 0

    async def _train_pump(self) -> None:
        step = 0
        while step < self.max_steps:
            self._evict_stale()
            producing = not (self._exhausted and not self._queue and "rollout" not in self._busy)
            local = self._step_size(len(self._ready), producing)
            finished = local == 0 and not producing
            # every rank decides on the same count (one all-reduce per poll, in lockstep)
            n, any_finished = await self._in_thread("train", self._agreed, local, finished) \
                if self.dp_group is not None else (local, finished)
            if n == 0:
                if any_finished:  # some rank can form no further step: the run ends everywhere
                    log.info("single controller: data exhausted after %d steps", step)
                    return
                await self._wait_wake(0.05)
                continue
            if n < self.groups_per_step:
                self.stats["shrunk_steps"] += 1
            keys = sorted(self._ready, key=lambda k: self._ready[k][0])[:n]   # oldest first
            groups, gids, vers = [], [], []
            for k in keys:
                ver, gid = self._ready.pop(k)
                groups.append(self.plane.get(self.PARTITION, k, timeout=30.0))
                self.plane.delete(self.PARTITION, k)
                gids.append(gid)
                vers.append(ver)
            self._notify()  # room in the buffer for the rollout pump
            t0 = time.perf_counter()
            metrics = await self._in_thread("train", self._train_locked, groups)
            self.version += 1
            step += 1
            if self.ledger is not None:
                self.ledger.mark_consumed([g for g in gids if g in self.ledger])
            self._dropped_since_step = 0
            m = dict(metrics or {})
            m.update({"step_time_s": time.perf_counter() - t0, "groups": float(n),
                      "avg_trajectory_age": float(sum(self.version - 1 - v for v in vers)) / max(1, n),
                      **{f"single_controller/{k}": float(v) for k, v in self.stats.items()},
                      **self.plane.metrics()})
            self.history.append(m)
            if self.on_step is not None:
                await self._in_thread("train", self.on_step, step, m)
            self._progress()
            self._notify()

    def _train_locked(self, groups: list):
        return self.train_fn(groups, self.version)

    async def _watchdog_loop(self) -> None:
        w = self.watchdog
        while not self._done:
            await asyncio.sleep(w.interval_s)
            now = time.monotonic()
            idle = now - self._last_progress
            long_calls = {p: now - t for p, t in self._busy.items() if now - t > w.stall_timeout_s}
            if idle > w.stall_timeout_s or long_calls:
                self.stats["stalls"] += 1
                what = (f"calls running for {', '.join(f'{p} {s:.1f}s' for p, s in long_calls.items())}"
                        if long_calls else f"no pump progress for {idle:.1f}s")
                log.warning("single controller stall: %s", what)
                if w.stall_action == "abort":
                    raise StallError(f"stall watchdog: {what} (stall_timeout_s={w.stall_timeout_s})")

    async def _main(self) -> None:
        from concurrent.futures import ThreadPoolExecutor

        # own worker threads (one per pump): an aborted run returns without joining
        # a call that is stuck; the thread ends with that call
        self._pool = ThreadPoolExecutor(max_workers=2, thread_name_prefix="single-controller")
        self._wake = asyncio.Event()
        self._progress()
        rollout = asyncio.create_task(self._rollout_pump(), name="rollout_pump")
        train = asyncio.create_task(self._train_pump(), name="train_pump")
        dog = asyncio.create_task(self._watchdog_loop(), name="watchdog")
        try:
            pending = {rollout, train, dog}
            while train in pending:
                done, pending = await asyncio.wait(pending, return_when=asyncio.FIRST_COMPLETED)
                for t in done:
                    if t.exception() is not None:
                        raise t.exception()
        finally:
            self._done = True
            self._notify()
            for t in (rollout, train, dog):
                t.cancel()
            await asyncio.gather(rollout, train, dog, return_exceptions=True)
            self._pool.shutdown(wait=False, cancel_futures=True)

    def run(self) -> list[dict]:
        """Run until ``max_steps`` training steps (or the data runs out); returns
        the per-step metrics."""
        asyncio.run(self._main())
        return self.history

    def state_dict(self) -> dict:
        """Controller state for a checkpoint: the version, counters, prompts
        waiting for a retry and the groups buffered in the plane."""
        return {"version": self.version, "stats": dict(self.stats),
                "queue": [{"gid": w.gid, "prompt": w.prompt, "attempts": dict(w.attempts)} for w in self._queue],
                "ready": {k: {"version": v, "gid": g, "batch": self.plane.get(self.PARTITION, k, timeout=5.0)}
                          for k, (v, g) in self._ready.items()}}

    def load_state_dict(self, sd: dict) -> None:
        self.version = int(sd["version"])
        self.stats.update(sd.get("stats", {}))
        self._queue = [_PromptWork(q["gid"], q["prompt"], dict(q["attempts"])) for q in sd.get("queue", [])]
        self._ready = {}
        for k, r in sd.get("ready", {}).items():
            self.plane.put(self.PARTITION, k, r["batch"])
            self._ready[k] = (int(r["version"]), r["gid"])


def _first_row(group, datum_rows) -> dict:
    """The prompt datum of a generated group (its first row's prompt message)."""
    log_ = group["message_log"][0]
    prompt = [m for m in log_ if m.get("role") != "assistant"][:1] or log_[:1]
    row = {"message_log": prompt, "task_name": group["task_name"][0] if "task_name" in group else "default",
           "extra_env_info": group["extra_env_info"][0] if "extra_env_info" in group else None,
           "length": int(sum(len(m["token_ids"]) for m in prompt)), "loss_multiplier": 1.0,
           "idx": int(group["idx"][0]) if "idx" in group else -1}
    return row


def single_controller_train(policy, dataloader, task_to_env: dict, master_config: dict, loss_fn=None, logger=None,
                            checkpointer=None, save_state=None, tokenizer=None, max_steps: Optional[int] = None,
                            data_plane=None, generate_fn: Optional[Callable] = None) -> dict:
    """Asynchronous GRPO through ``SingleController`` (config ``grpo.single_controller``
    with the options named in the module docstring; the trajectory age bound is
    ``grpo.async_grpo.max_trajectory_age_steps``).  ``generate_fn`` replaces the
    multi-turn rollout (tests use it to inject failures and delays)."""
    from rl_b200.algorithms.advantage_estimator import make_advantage_estimator
    from rl_b200.algorithms.async_utils import groups_to_batch
    from rl_b200.algorithms.grpo import DEFAULT_GRPO_CONFIG, GRPOSaveState, build_train_data
    from rl_b200.algorithms.loss.loss_functions import ClippedPGLossFn
    from rl_b200.algorithms.utils import set_seed
    from rl_b200.experience.rollouts import run_multi_turn_rollout

    ps = policy.ps
    if ps.tp_size > 1:
        raise NotImplementedError("the single controller generates in a worker thread and needs TP=1 generation")
    cfg = {**DEFAULT_GRPO_CONFIG, **master_config.get("grpo", {})}
    scfg = dict(cfg.get("single_controller") or {})
    acfg = {**DEFAULT_GRPO_CONFIG["async_grpo"], **(cfg.get("async_grpo") or {})}
    loss_cfg = master_config.get("loss_fn", {})
    loss_fn = loss_fn or ClippedPGLossFn(loss_cfg)
    adv_cfg = dict(cfg.get("adv_estimator", {}) or {})
    adv_cfg.setdefault("normalize_rewards", cfg["normalize_rewards"])
    adv_cfg.setdefault("use_leave_one_out_baseline", cfg["use_leave_one_out_baseline"])
    estimator = make_advantage_estimator(adv_cfg, loss_cfg)
    G = int(cfg["num_generations_per_prompt"])
    n_groups = max(1, int(cfg["num_prompts_per_step"]) // max(1, ps.dp_size))
    max_seq = int(master_config["policy"]["max_total_sequence_length"])
    kl_on = float(loss_cfg.get("reference_policy_kl_penalty", 0.0) or 0.0) != 0.0
    state = save_state or GRPOSaveState.default()
    start = int(state["current_step"])
    max_steps = max_steps if max_steps is not None else int(cfg["max_num_steps"])
    set_seed(int(cfg["seed"]) + ps.dp_rank)
    engine = getattr(policy, "engine", None)
    if engine is not None:
        engine.capture_error_mode = "thread_local"
        engine.kv_arena = None  # training runs meanwhile: the KV cache may not borrow its arena
    weights_lock = threading.RLock()

    def default_generate(batch, version):
        n = len(batch["message_log"]) // G
        base = version * 1_000_000 + ps.dp_rank * 10_000
        batch["group_id"] = torch.arange(base, base + n).repeat_interleave(G)
        policy.prepare_for_generation(len(batch["message_log"]))
        rollout, _ = run_multi_turn_rollout(policy, batch, tokenizer, task_to_env, max_seq,
                                            int(cfg["max_rollout_turns"]))
        return rollout

    def train_fn(groups, version):
        rollout = groups_to_batch(groups)
        gids = torch.arange(len(groups)).repeat_interleave(G)
        train_data, adv_stats = build_train_data(rollout, estimator, cfg, loss_cfg, gids)
        policy.prepare_for_lp_inference()
        train_data["prev_logprobs"] = policy.get_logprobs(train_data)["logprobs"]
        if kl_on:
            train_data["reference_policy_logprobs"] = \
                policy.get_reference_policy_logprobs(train_data)["reference_logprobs"]
        policy.prepare_for_training()
        st = policy.begin_train_step(train_data, loss_fn)
        for i in range(st.num_microbatches):
            policy.train_microbatch(st, i)
        with weights_lock:  # no rollout generates from a half-updated model
            res = policy.finish_train_step(st)
            policy.refit()
        out = dict(res)
        out.update(adv_stats)
        out["total_tokens"] = float(train_data["input_lengths"].sum())
        return out

    def on_step(step, metrics):
        state["current_step"] = start + step
        state["total_steps"] = int(state.get("total_steps", 0)) + 1
        state["consumed_samples"] = int(state.get("consumed_samples", 0)) + int(metrics["groups"]) * ps.dp_size
        if logger:
            logger.log_metrics(metrics, start + step, prefix="train")
        if checkpointer is not None and checkpointer.should_save(start + step):
            with weights_lock:
                checkpointer.save(policy, state, dataloader, metrics, start + step,
                                  rank_files={_controller_file(): sc.state_dict()})

    sc = SingleController(generate_fn or default_generate, train_fn, dataloader, G, n_groups,
                          max(0, max_steps - start), cfg=scfg, data_plane=data_plane, initial_version=start,
                          max_trajectory_age_steps=int(acfg.get("max_trajectory_age_steps", 1)),
                          dp_group=ps.dp_group if ps.dp_size > 1 else None, weights_lock=weights_lock,
                          on_step=on_step)
    if checkpointer is not None and checkpointer.get_latest_checkpoint_path():
        import os

        f = os.path.join(checkpointer.get_latest_checkpoint_path(), _controller_file())
        if os.path.exists(f):
            sc.load_state_dict(torch.load(f, weights_only=False))
    sc.run()
    state["single_controller"] = dict(sc.stats)
    return state


def _controller_file() -> str:
    import torch.distributed as dist

    return f"single_controller_rank{dist.get_rank() if dist.is_initialized() else 0}.pt"
