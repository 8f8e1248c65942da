"""Generation-fleet state machine, selector and supervisor (host only)."""

import pytest

from rl_b200.models.generation.fleet_health import (EngineSupervisor, FleetHealthPolicy, GenerationFleetExhausted,
                                                    GenerationFleetHealth, HealthyShardSelector, ShardState)


def test_probe_failures_suspect_then_dead_and_recovery_needs_refit():
    f = GenerationFleetHealth(3, FleetHealthPolicy(unhealthy_threshold=2, healthy_threshold=2))
    f.record_probe(0, ok=False)
    assert f.state_of(0) == ShardState.SUSPECT and 0 in f.serving_shards()
    f.record_probe(0, ok=True)
    f.record_probe(0, ok=True)
    assert f.state_of(0) == ShardState.HEALTHY
    f.record_probe(1, ok=False)
    f.record_probe(1, ok=False)
    assert f.state_of(1) == ShardState.DEAD and f.absent_shards() == [1]
    epoch = f.membership_epoch
    # probes never revive a dead shard
    f.record_probe(1, ok=True)
    assert f.state_of(1) == ShardState.DEAD
    assert f.mark_restarting(1) and f.state_of(1) == ShardState.RESTARTING
    f.mark_loaded(1)
    assert f.state_of(1) == ShardState.STALE and 1 not in f.serving_shards()
    assert f.membership_epoch == epoch + 1  # back among the refit participants
    f.set_trainer_version(7)
    f.report_refit(1, 6)
    assert f.state_of(1) == ShardState.STALE
    f.report_refit(1, 7)
    assert f.state_of(1) == ShardState.HEALTHY


def test_reported_failures_not_cleared_by_probes_and_retirement():
    f = GenerationFleetHealth(2, FleetHealthPolicy(unhealthy_threshold=2, max_restart_attempts_per_shard=1,
                                                   min_healthy_shards=1))
    f.report_failure(0, RuntimeError("wedged"))
    f.record_probe(0, ok=True)
    f.record_probe(0, ok=True)
    assert f.state_of(0) == ShardState.SUSPECT  # a wedged engine that answers probes stays suspect
    f.report_failure(0, "again")
    assert f.state_of(0) == ShardState.DEAD
    assert f.mark_restarting(0)
    f.mark_restart_failed(0, "boom")
    assert f.state_of(0) == ShardState.RETIRED
    f.record_death(1)
    with pytest.raises(GenerationFleetExhausted):
        f.raise_if_exhausted()


def test_selector_least_inflight_and_supervisor_restarts():
    f = GenerationFleetHealth(3)
    sel = HealthyShardSelector(f)
    picks = []
    for _ in range(3):
        i = sel.next_shard()
        sel.acquire(i)
        picks.append(i)
    assert sorted(picks) == [0, 1, 2]
    sel.release(1)
    assert sel.next_shard() == 1
    f.record_death(2)
    calls = []

    def restart(i):
        calls.append(i)
        if len(calls) == 1:
            raise RuntimeError("first restart fails")

    sup = EngineSupervisor(f, restart)
    sup.tick()
    sup.join()
    assert f.state_of(2) == ShardState.DEAD and sup.restarts_failed == 1
    sup.tick()
    sup.join()
    assert f.state_of(2) == ShardState.STALE and sup.restarts_ok == 1 and calls == [2, 2]
    assert 2 not in f.serving_shards()


def test_supervisor_recreates_a_dead_engine_through_the_policy():
    """A generation shard reported dead is rebuilt by the supervisor through
    ``Policy.recreate_worker``: the new engine serves the same greedy rollouts
    and the shard returns to serving after the refit."""
    import torch

    from rl_b200.distributed.batched_data_dict import BatchedDataDict
    from rl_b200.models.config import get_model_config
    from rl_b200.models.generation.fleet_health import EngineSupervisor, GenerationFleetHealth, ShardState
    from rl_b200.models.policy.lm_policy import Policy
    from rl_b200.models.policy.worker import PolicyWorker

    pcfg = {"max_total_sequence_length": 48, "precision": "float32", "train_global_batch_size": 4,
            "generation": {"temperature": 1.0, "max_new_tokens": 6}}
    pol = Policy(PolicyWorker(pcfg, model_cfg=get_model_config("tiny-llama"), seed=2))
    data = BatchedDataDict({"input_ids": torch.randint(0, 512, (4, 10), generator=torch.Generator().manual_seed(1)),
                            "input_lengths": torch.tensor([10, 7, 9, 3])})
    before = pol.generate(data, greedy=True)["output_ids"]
    old = pol.worker.engine
    fleet = GenerationFleetHealth(1)
    sup = EngineSupervisor(fleet, lambda i: pol.recreate_worker(i))
    fleet.record_death(0, "engine crashed")
    sup.tick()
    sup.join()
    assert pol.worker.engine is not old and pol.worker.engine_incarnation == 1
    assert sup.restarts_ok == 1 and fleet.state_of(0) != ShardState.DEAD
    fleet.report_refit(0, fleet.trainer_version if hasattr(fleet, "trainer_version") else 0)
    after = pol.generate(data, greedy=True)["output_ids"]
    assert torch.equal(before, after)
    assert pol.sharding_annotations.get_axis_size("data_parallel") == 1
