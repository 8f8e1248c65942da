"""Binary codec for ``BatchedDataDict`` payloads: a JSON header (per field:
kind, dtype, shape, byte range) followed by the raw tensor bytes; non-tensor
fields (lists of strings, dicts, ...) are pickled.  Optional zlib compression
of the body."""

from __future__ import annotations

import json
import pickle
import struct
import zlib

import numpy as np
import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["encode_batch", "decode_batch"]

_MAGIC = b"RLDP"


def encode_batch(batch: dict, compress: bool = False) -> bytes:
    fields, chunks, off = [], [], 0
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            t = v.detach().cpu().contiguous()
            raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
            fields.append({"k": k, "t": "tensor", "dtype": str(t.dtype).replace("torch.", ""),
                           "shape": list(t.shape), "o": off, "n": len(raw)})
        else:
            raw = pickle.dumps(v, protocol=pickle.HIGHEST_PROTOCOL)
            fields.append({"k": k, "t": "pickle", "o": off, "n": len(raw)})
        chunks.append(raw)
        off += len(raw)
    body = b"".join(chunks)
    if compress:
        body = zlib.compress(body, 1)
    head = json.dumps({"fields": fields, "z": compress}).encode()
    return _MAGIC + struct.pack("<I", len(head)) + head + body


def decode_batch(blob: bytes) -> BatchedDataDict:
    if blob[:4] != _MAGIC:
        raise ValueError("not a data-plane payload")
    (hl,) = struct.unpack("<I", blob[4:8])
    head = json.loads(blob[8:8 + hl].decode())
    body = blob[8 + hl:]
    if head["z"]:
        body = zlib.decompress(body)
    out = BatchedDataDict()
    for f in head["fields"]:
        raw = body[f["o"]:f["o"] + f["n"]]
        if f["t"] == "tensor":
            dt = getattr(torch, f["dtype"])
            if f["n"]:
                u8 = torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy())
                out[f["k"]] = u8.view(dt).reshape(f["shape"])
            else:
                out[f["k"]] = torch.empty(f["shape"], dtype=dt)
        else:
            out[f["k"]] = pickle.loads(raw)
    return out
