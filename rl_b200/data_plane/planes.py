"""Data-plane backends.

``put(partition, key, batch)`` / ``get(partition, key, timeout)`` /
``delete`` / ``keys`` with per-plane observability counters (ops, bytes,
seconds).  ``InProcessDataPlane`` keeps encoded payloads in a dict (threads of
one process, e.g. the async rollout pump and the trainer);
``StoreDataPlane`` keeps them in a ``torch.distributed`` key-value store
(``TCPStore``; every process of the job, or of two jobs - rollout and
training - that share the store) so a producer rank's samples can be consumed
by any other rank.  ``get`` blocks (bounded by ``timeout``) until the key exists.
"""

from __future__ import annotations

import threading
import time
from datetime import timedelta
from typing import Optional

from rl_b200.data_plane.codec import decode_batch, encode_batch
from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["DataPlane", "InProcessDataPlane", "StoreDataPlane", "create_data_plane"]


class DataPlane:
    def __init__(self, compress: bool = False):
        self.compress = compress
        self.stats = {"puts": 0, "gets": 0, "bytes_put": 0, "bytes_get": 0, "put_s": 0.0, "get_s": 0.0}

    # backend hooks
    def _set(self, key: str, blob: bytes) -> None:
        raise NotImplementedError

    def _get(self, key: str, timeout: float) -> bytes:
        raise NotImplementedError

    def _del(self, key: str) -> None:
        raise NotImplementedError

    def keys(self, partition: str) -> list[str]:
        raise NotImplementedError

    # public API
    def put(self, partition: str, key: str, batch: dict) -> None:
        t0 = time.perf_counter()
        blob = encode_batch(batch, self.compress)
        self._set(f"{partition}/{key}", blob)
        self.stats["puts"] += 1
        self.stats["bytes_put"] += len(blob)
        self.stats["put_s"] += time.perf_counter() - t0

    def get(self, partition: str, key: str, timeout: float = 60.0) -> BatchedDataDict:
        t0 = time.perf_counter()
        blob = self._get(f"{partition}/{key}", timeout)
        out = decode_batch(blob)
        self.stats["gets"] += 1
        self.stats["bytes_get"] += len(blob)
        self.stats["get_s"] += time.perf_counter() - t0
        return out

    def delete(self, partition: str, key: str) -> None:
        self._del(f"{partition}/{key}")

    def metrics(self) -> dict:
        return {f"data_plane/{k}": float(v) for k, v in self.stats.items()}


class InProcessDataPlane(DataPlane):
    def __init__(self, compress: bool = False):
        super().__init__(compress)
        self._d: dict[str, bytes] = {}
        self._cv = threading.Condition()

    def _set(self, key, blob):
        with self._cv:
            self._d[key] = blob
            self._cv.notify_all()

    def _get(self, key, timeout):
        with self._cv:
            if not self._cv.wait_for(lambda: key in self._d, timeout=timeout):
                raise TimeoutError(f"data plane: {key!r} not produced within {timeout} s")
            return self._d[key]

    def _del(self, key):
        with self._cv:
            self._d.pop(key, None)

    def keys(self, partition):
        with self._cv:
            return sorted(k.split("/", 1)[1] for k in self._d if k.startswith(partition + "/"))


class StoreDataPlane(DataPlane):
    """Over a ``torch.distributed`` Store (default: the job's TCPStore at
    MASTER_ADDR / a dedicated port).  Key listing is kept in an index key per
    partition (append-only, ``\\n``-separated)."""

    def __init__(self, store=None, host: str = "127.0.0.1", port: int = 0, is_master: bool = False,
                 world_size: Optional[int] = None, compress: bool = False, prefix: str = "rldp"):
        super().__init__(compress)
        import torch.distributed as dist

        if store is None:
            store = dist.TCPStore(host, port, world_size, is_master, timedelta(seconds=300), wait_for_workers=False)
        self.store = dist.PrefixStore(prefix, store)

    def _set(self, key, blob):
        self.store.set(key, blob)
        part, k = key.split("/", 1)
        self.store.append(f"__index__/{part}", (k + "\n").encode())

    def _get(self, key, timeout):
        self.store.wait([key], timedelta(seconds=timeout))
        return bytes(self.store.get(key))

    def _del(self, key):
        self.store.delete_key(key)

    def keys(self, partition):
        idx = f"__index__/{partition}"
        if not self.store.check([idx]):
            return []
        names = [k for k in bytes(self.store.get(idx)).decode().split("\n") if k]
        return sorted({k for k in names if self.store.check([f"{partition}/{k}"])})


def create_data_plane(cfg: Optional[dict], store=None) -> Optional[DataPlane]:
    """``{"enabled": bool, "backend": "in_process" | "store", "compress": bool}``."""
    if not cfg or not cfg.get("enabled", False):
        return None
    backend = str(cfg.get("backend", "in_process"))
    if backend == "in_process":
        return InProcessDataPlane(bool(cfg.get("compress", False)))
    if backend == "store":
        return StoreDataPlane(store=store, host=cfg.get("host", "127.0.0.1"), port=int(cfg.get("port", 0)),
                              is_master=bool(cfg.get("is_master", False)), compress=bool(cfg.get("compress", False)))
    raise ValueError(f"unknown data plane backend {backend!r}")
