"""Key-value sample store between producers (rollout) and consumers (training).

Reference: the TransferQueue data plane (``nemo_rl/data_plane/interfaces.py``,
``factory.py``, ``codec.py``, ``observability.py``)."""

from rl_b200.data_plane.codec import decode_batch, encode_batch
from rl_b200.data_plane.planes import DataPlane, InProcessDataPlane, StoreDataPlane, create_data_plane

__all__ = ["DataPlane", "InProcessDataPlane", "StoreDataPlane", "create_data_plane", "encode_batch", "decode_batch"]
