"""Checkpoint engines: bucketed point-to-point weight transfer from a policy
process to a rollout process that shares no process group with it.

Reference: ``nemo_rl/utils/checkpoint_engines/base.py`` (``CheckpointEngine``:
``prepare`` returns serialisable metadata, ``init_policy_process_group`` /
``init_rollout_process_group`` connect the two sides from each other's metadata,
``send_weights`` / ``receive_weight_batches`` move ``(name, tensor)`` weights in
buckets of ``bucket_size`` bytes, ``finalize`` releases per-refit state;
``split_weight_chunks`` / ``merge_weight_chunk_batches`` cut tensors larger than
a bucket into byte chunks and glue them back; ``create_checkpoint_engine`` picks
a backend by name or ``module:Class``) and its NIXL backend (``nixl.py``).

Backends here, both single-node:

* ``shm``  - two POSIX shared-memory slots of ``bucket_size`` bytes; the sender
  fills a slot (pinned-host staging of device tensors) and publishes the slot's
  tensor metadata under a sequence number in a key-value store; the receiver
  copies the slot out (to ``device``) and acknowledges.  Needs no GPU.
* ``cuda_ipc`` - the same protocol with the two slots in the SENDER's device
  memory, exported by CUDA IPC: the receiver's copy-out is a device-to-device
  copy over NVLink from the peer GPU (or within one GPU), with no host staging.

Flow control: slot ``s = seq % 2`` may be refilled once the receiver
acknowledged ``seq - 2``; every wait polls the store with a deadline
(``timeout_s``) and raises ``TimeoutError`` instead of hanging.
"""

from __future__ import annotations

import abc
import importlib
import pickle
import time
from dataclasses import dataclass
from datetime import timedelta
from typing import Any, Iterable, Iterator, Optional

import torch

__all__ = ["TensorMeta", "CheckpointEngine", "SharedMemoryCheckpointEngine", "CudaIpcCheckpointEngine",
           "CheckpointEngineSynchronizer", "create_checkpoint_engine", "split_weight_chunks",
           "merge_weight_chunk_batches"]


@dataclass
class TensorMeta:
    name: str
    shape: torch.Size
    dtype: torch.dtype
    chunk_offset: int      # byte offset of this chunk inside the tensor
    chunk_size: int        # bytes of this chunk
    offset: Optional[int]  # byte offset of the chunk inside the bucket

    @property
    def nbytes(self) -> int:
        return int(torch.Size(self.shape).numel()) * torch.empty((), dtype=self.dtype).element_size()


def split_weight_chunks(weights: Iterable[tuple[str, torch.Tensor]], bucket_size: int
                        ) -> Iterator[tuple[TensorMeta, torch.Tensor]]:
    """``(name, tensor)`` -> ``(meta, uint8 chunk)`` with chunks of at most ``bucket_size`` bytes."""
    for name, w in weights:
        flat = w.detach().contiguous().view(-1).view(torch.uint8)
        n = flat.numel()
        for c0 in range(0, max(n, 1), bucket_size):
            size = min(bucket_size, n - c0)
            yield TensorMeta(name, w.shape, w.dtype, c0, size, None), flat[c0:c0 + size]


def merge_weight_chunk_batches(batches: Iterable[list[tuple[TensorMeta, torch.Tensor]]],
                               device: Optional[torch.device] = None) -> Iterator[list[tuple[str, torch.Tensor]]]:
    """Inverse of ``split_weight_chunks`` over received batches: whole tensors
    pass through; a chunked tensor is assembled and emitted with the batch that
    completes it."""
    pending: Optional[torch.Tensor] = None
    for batch in batches:
        out = []
        for meta, chunk in batch:
            if meta.chunk_offset == 0 and meta.chunk_size == meta.nbytes:
                out.append((meta.name, chunk.view(meta.dtype).view(meta.shape)))
                continue
            if meta.chunk_offset == 0:
                pending = torch.empty(meta.nbytes, dtype=torch.uint8, device=device or chunk.device)
            assert pending is not None, f"chunk of {meta.name} arrived without its first chunk"
            pending[meta.chunk_offset:meta.chunk_offset + meta.chunk_size].copy_(chunk)
            if meta.chunk_offset + meta.chunk_size == meta.nbytes:
                out.append((meta.name, pending.view(meta.dtype).view(meta.shape)))
                pending = None
        if out:
            yield out


class CheckpointEngine(abc.ABC):
    """Transport interface (names as in the reference; synchronous generators)."""

    def get_target_weight_layout(self) -> Optional[dict]:
        return None

    @abc.abstractmethod
    def prepare(self) -> Any:
        """Allocate resources; returns metadata the peer side needs."""

    @abc.abstractmethod
    def init_policy_process_group(self, *, worker_rank: int, train_world_size: int, rollout_world_size: int,
                                  metadata: list) -> None:
        """Connect the policy side (``metadata``: every side's ``prepare`` result)."""

    @abc.abstractmethod
    def init_rollout_process_group(self, *, rollout_rank: int, train_world_size: int, rollout_world_size: int,
                                   metadata: list) -> None:
        """Connect the rollout side."""

    def finalize(self) -> None:
        """Release per-refit state."""

    @abc.abstractmethod
    def send_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> int:
        """Send ``(name, tensor)`` weights; returns the bytes sent."""

    @abc.abstractmethod
    def receive_weight_batches(self) -> Iterator[list[tuple[str, torch.Tensor]]]:
        """Yield ``(name, tensor)`` batches until the sender's end marker."""


class _SlotEngine(CheckpointEngine):
    """Two-slot bucket protocol over a key-value store (``torch.distributed``
    Store); subclasses provide the slots and the copy into / out of them."""

    def __init__(self, bucket_size: int = 256 << 20, store=None, prefix: str = "ckpt_engine",
                 timeout_s: float = 300.0, device: Optional[str] = None, host: str = "127.0.0.1", port: int = 0,
                 is_master: bool = False):
        self.bucket_size = int(bucket_size)
        self._store_args = (store, host, port, is_master)
        self.prefix = prefix
        self.timeout_s = float(timeout_s)
        self.device = torch.device(device) if device else None
        self.store = None
        self.seq = 0          # buckets sent / received in this engine's lifetime
        self.refit = 0

    # ----------------------------------------------------------- wiring
    def _connect(self) -> None:
        import torch.distributed as dist

        store, host, port, is_master = self._store_args
        if store is None:
            store = dist.TCPStore(host, port, None, is_master, timedelta(seconds=self.timeout_s),
                                  wait_for_workers=False)
        self.port = getattr(store, "port", port)  # where the other side connects (a master picks it when 0)
        self.store = dist.PrefixStore(self.prefix, store)

    def _key(self, *parts) -> str:
        return "/".join(str(p) for p in parts)

    def _wait_key(self, key: str) -> bytes:
        deadline = time.monotonic() + self.timeout_s
        while not self.store.check([key]):
            if time.monotonic() > deadline:
                raise TimeoutError(f"checkpoint engine: {key!r} not published within {self.timeout_s:.0f} s")
            time.sleep(0.0005)
        return bytes(self.store.get(key))

    # ------------------------------------------------------------- slots
    @abc.abstractmethod
    def _slot_write(self, slot: int, offset: int, chunk: torch.Tensor) -> None: ...

    @abc.abstractmethod
    def _slot_read(self, slot: int, offset: int, nbytes: int) -> torch.Tensor: ...

    def _slot_fence(self) -> None:
        """Make the slot writes of a bucket visible before it is published."""

    # -------------------------------------------------------------- send
    def send_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> int:
        sent, used, metas = 0, 0, []
        claimed = False  # the current slot's previous bucket was acknowledged

        def claim():
            if self.seq >= 2:
                self._wait_key(self._key("ack", self.seq - 2))

        def publish(last: bool):
            nonlocal used, metas, claimed
            if not claimed:
                claim()
            self._slot_fence()
            self.store.set(self._key("meta", self.seq), pickle.dumps((metas, last)))
            self.seq += 1
            used, metas, claimed = 0, [], False

        for meta, chunk in split_weight_chunks(weights, self.bucket_size):
            if metas and used + meta.chunk_size > self.bucket_size:
                publish(False)
            if not claimed:
                claim()
                claimed = True
            meta.offset = used
            self._slot_write(self.seq % 2, used, chunk)
            metas.append(meta)
            used += (meta.chunk_size + 255) // 256 * 256  # chunk starts stay 256-byte aligned
            sent += meta.chunk_size
        publish(True)
        self.refit += 1
        return sent

    # ----------------------------------------------------------- receive
    def _received_batches(self) -> Iterator[list[tuple[TensorMeta, torch.Tensor]]]:
        while True:
            seq = self.seq
            metas, last = pickle.loads(self._wait_key(self._key("meta", seq)))
            slot = seq % 2
            batch = [(m, self._slot_read(slot, m.offset, m.chunk_size)) for m in metas]
            self.seq += 1
            self.store.set(self._key("ack", seq), b"1")  # copies are complete: the slot may be reused
            if batch:
                yield batch
            if last:
                self.refit += 1
                return

    def receive_weight_batches(self) -> Iterator[list[tuple[str, torch.Tensor]]]:
        yield from merge_weight_chunk_batches(self._received_batches(), self.device)


class SharedMemoryCheckpointEngine(_SlotEngine):
    """POSIX shared-memory slots (``multiprocessing.shared_memory``)."""

    def __init__(self, bucket_size: int = 256 << 20, **kw):
        super().__init__(bucket_size, **kw)
        self._shm = None
        self._name: Optional[str] = None

    def prepare(self) -> dict:
        from multiprocessing import shared_memory

        self._shm = shared_memory.SharedMemory(create=True, size=2 * self.bucket_size)
        self._name = self._shm.name
        return {"backend": "shm", "name": self._name, "bucket_size": self.bucket_size}

    def init_policy_process_group(self, *, worker_rank: int, train_world_size: int, rollout_world_size: int,
                                  metadata: list) -> None:
        self._connect()

    def init_rollout_process_group(self, *, rollout_rank: int, train_world_size: int, rollout_world_size: int,
                                   metadata: list) -> None:
        from multiprocessing import shared_memory

        src = metadata[rollout_rank % max(1, train_world_size)]
        self.bucket_size = int(src["bucket_size"])
        self._shm = shared_memory.SharedMemory(name=src["name"])
        self._connect()

    def _view(self) -> torch.Tensor:
        return torch.frombuffer(self._shm.buf, dtype=torch.uint8)

    def _slot_write(self, slot, offset, chunk):
        base = slot * self.bucket_size + offset
        self._view()[base:base + chunk.numel()].copy_(chunk.cpu())

    def _slot_read(self, slot, offset, nbytes):
        base = slot * self.bucket_size + offset
        out = self._view()[base:base + nbytes].clone()
        return out.to(self.device) if self.device is not None else out

    def finalize(self) -> None:
        pass

    def close(self, unlink: bool = False) -> None:
        if self._shm is not None:
            self._shm.close()
            if unlink:
                self._shm.unlink()
            self._shm = None


class CudaIpcCheckpointEngine(_SlotEngine):
    """Slots in the sender's device memory, opened by the receiver through CUDA IPC."""

    def __init__(self, bucket_size: int = 256 << 20, **kw):
        super().__init__(bucket_size, **kw)
        self._ptr = None
        self._slots: Optional[torch.Tensor] = None
        self._opened = None

    def prepare(self) -> dict:
        from rl_b200.ops._ext import ext

        ptr, handle = ext().symm_alloc(2 * self.bucket_size)
        self._ptr = int(ptr)
        self._slots = ext().symm_view(self._ptr, 2 * self.bucket_size, 0, torch.cuda.current_device())
        return {"backend": "cuda_ipc", "handle": bytes(handle.numpy().tobytes()), "bucket_size": self.bucket_size}

    def init_policy_process_group(self, *, worker_rank: int, train_world_size: int, rollout_world_size: int,
                                  metadata: list) -> None:
        self._connect()

    def init_rollout_process_group(self, *, rollout_rank: int, train_world_size: int, rollout_world_size: int,
                                   metadata: list) -> None:
        from rl_b200.ops._ext import ext

        src = metadata[rollout_rank % max(1, train_world_size)]
        self.bucket_size = int(src["bucket_size"])
        self._opened = int(ext().symm_open(torch.frombuffer(bytearray(src["handle"]), dtype=torch.uint8)))
        self._slots = ext().symm_view(self._opened, 2 * self.bucket_size, 0, torch.cuda.current_device())
        if self.device is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._connect()

    def _slot_write(self, slot, offset, chunk):
        base = slot * self.bucket_size + offset
        self._slots[base:base + chunk.numel()].copy_(chunk, non_blocking=True)

    def _slot_fence(self) -> None:
        torch.cuda.current_stream().synchronize()  # the bucket is in the slot before it is published

    def _slot_read(self, slot, offset, nbytes):
        base = slot * self.bucket_size + offset
        out = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        out.copy_(self._slots[base:base + nbytes])
        torch.cuda.current_stream().synchronize()  # copied out before the slot is acknowledged
        return out

    def close(self) -> None:
        from rl_b200.ops._ext import ext

        if self._opened is not None:
            ext().symm_close(self._opened)
            self._opened = None
        if self._ptr is not None:
            ext().symm_close(self._ptr)
            self._ptr = None
        self._slots = None


_BACKENDS = {"shm": SharedMemoryCheckpointEngine, "cuda_ipc": CudaIpcCheckpointEngine,
             # the reference's RDMA backend: on one node the same peer-to-peer role is CUDA IPC
             "nixl": CudaIpcCheckpointEngine}


def create_checkpoint_engine(backend: str, *, bucket_size_bytes: int, engine_kwargs: Optional[dict] = None
                             ) -> CheckpointEngine:
    """``backend``: ``shm``, ``cuda_ipc`` (``nixl`` maps to it on one node) or ``module:Class``."""
    kw = dict(engine_kwargs or {})
    if backend in _BACKENDS:
        return _BACKENDS[backend](bucket_size_bytes, **kw)
    if ":" not in backend:
        raise ValueError(f"unknown checkpoint-engine backend {backend!r}: {sorted(_BACKENDS)} or 'module:Class'")
    mod, cls = backend.split(":", 1)
    return getattr(importlib.import_module(mod), cls)(bucket_size=bucket_size_bytes, **kw)


class CheckpointEngineSynchronizer:
    """Weight synchronizer over a checkpoint engine for a policy and a rollout
    process that share no process group: the policy side sends the model's
    HF-named weights (``sync``), the rollout side loads every received batch into
    its model by name (``receive_into``)."""

    name = "checkpoint_engine"

    def __init__(self, engine: CheckpointEngine, model=None):
        self.engine = engine
        self.model = model
        self.version = 0
        self.stats: dict = {"syncs": 0, "last_s": 0.0, "bytes": 0}

    def sync(self) -> dict:
        from rl_b200.models.checkpoint_io import hf_state_dict

        t0 = time.perf_counter()
        nbytes = self.engine.send_weights(hf_state_dict(self.model, dtype=None).items())
        self.version += 1
        self.stats.update(syncs=self.stats["syncs"] + 1, last_s=time.perf_counter() - t0, bytes=int(nbytes))
        return dict(self.stats, version=self.version)

    def receive_into(self, model) -> int:
        """Receive one refit into ``model``; returns the number of tensors loaded."""
        from rl_b200.models.checkpoint_io import load_hf_state_dict

        sd: dict = {}
        for batch in self.engine.receive_weight_batches():
            sd.update(batch)  # fused parameters (qkv, gate / up) need all their parts
        load_hf_state_dict(model, sd)
        self.version += 1
        return len(sd)

    def shutdown(self) -> None:
        close = getattr(self.engine, "close", None)
        if close is not None:
            close()
