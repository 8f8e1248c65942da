"""Train -> rollout weight synchronisation (refit) transports."""

from rl_b200.weight_sync.colocated import ColocatedInPlaceSynchronizer, ColocatedReshardSynchronizer
from rl_b200.weight_sync.interfaces import WeightSynchronizer

__all__ = ["WeightSynchronizer", "ColocatedInPlaceSynchronizer", "ColocatedReshardSynchronizer",
           "create_weight_synchronizer"]

# reference refit_transport names -> transports here
_ALIASES = {"vllm_s3_sparse": "sparse_broadcast", "vllm_zmq_sparse": "sparse_broadcast", "nccl": "broadcast",
            "ipc": "inplace", "cuda_ipc": "inplace", "nccl_reshard": "reshard"}


def create_weight_synchronizer(kind: str, **kwargs) -> WeightSynchronizer:
    """Synchronizer ``kind`` (``inplace`` / ``reshard`` / ``broadcast`` /
    ``sparse_broadcast``, or a reference ``refit_transport`` name) built from the
    transport's constructor arguments."""
    from rl_b200.weight_sync.broadcast import PackedBroadcastSynchronizer, SparseDeltaBroadcastSynchronizer

    table = {"inplace": ColocatedInPlaceSynchronizer, "reshard": ColocatedReshardSynchronizer,
             "broadcast": PackedBroadcastSynchronizer, "sparse_broadcast": SparseDeltaBroadcastSynchronizer}
    name = _ALIASES.get(kind, kind)
    if name not in table:
        raise ValueError(f"unknown weight synchronizer {kind!r}; known: {sorted(table)} + {sorted(_ALIASES)}")
    return table[name](**kwargs)
