"""Train -> rollout weight synchronisation (refit) transports."""

from rl_b200.weight_sync.colocated import ColocatedInPlaceSynchronizer, ColocatedReshardSynchronizer
from rl_b200.weight_sync.interfaces import WeightSynchronizer

__all__ = ["WeightSynchronizer", "ColocatedInPlaceSynchronizer", "ColocatedReshardSynchronizer"]
