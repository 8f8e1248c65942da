"""Flattening of message logs into model inputs and per-token masks.

Reference: ``batched_message_log_to_flat_message`` (``nemo_rl/data/llm_message_utils.py:288``)
and the helpers around it (``get_keys_from_message_log``, ``add_loss_mask_to_message_log``).
The flat form is right-padded ``[B, S]`` tensors plus ``input_lengths``; per-message
fields (``token_loss_mask``, ``generation_logprobs``) are concatenated the same way.
"""

from __future__ import annotations

from typing import Optional

import torch

from rl_b200.distributed.batched_data_dict import BatchedDataDict

__all__ = ["message_log_to_flat", "batched_message_log_to_flat_message", "add_loss_mask_to_message_log",
           "get_keys_from_message_log"]


def add_loss_mask_to_message_log(message_logs: list[list[dict]], roles_to_train_on: tuple = ("assistant",),
                                 only_unmask_final: bool = False) -> None:
    """Set ``token_loss_mask`` on every message: ones for trained roles, else zeros."""
    for log in message_logs:
        for i, msg in enumerate(log):
            train = msg["role"] in roles_to_train_on and (not only_unmask_final or i == len(log) - 1)
            n = len(msg["token_ids"])
            msg["token_loss_mask"] = torch.ones(n, dtype=torch.int64) if train else torch.zeros(n, dtype=torch.int64)


def get_keys_from_message_log(log: list[dict], keys: list[str]) -> list[dict]:
    return [{k: m[k] for k in keys if k in m} for m in log]


# per-token fields whose "missing" value is not zero
PAD_VALUES = {"routed_experts": -1}


def message_log_to_flat(log: list[dict]) -> dict[str, torch.Tensor]:
    """Concatenate the per-token fields of a message log (tensors whose first
    dimension is the message's token count; trailing dimensions are kept, e.g.
    ``routed_experts [L, layers, top_k]``)."""
    out: dict[str, list] = {}
    n = 0
    for msg in log:
        L = len(msg["token_ids"])
        n += L
        for k, v in msg.items():
            if isinstance(v, torch.Tensor) and v.dim() >= 1 and v.shape[0] == L:
                out.setdefault(k, []).append(v)
    flat = {k: torch.cat(v) for k, v in out.items()}
    # keys missing on some messages: fill with the key's pad value
    for k in list(flat.keys()):
        if flat[k].shape[0] != n:
            parts = []
            for msg in log:
                L = len(msg["token_ids"])
                parts.append(msg[k] if k in msg else
                             torch.full((L,) + tuple(flat[k].shape[1:]), PAD_VALUES.get(k, 0), dtype=flat[k].dtype))
            flat[k] = torch.cat(parts)
    return flat


def batched_message_log_to_flat_message(message_logs: list[list[dict]], pad_value_dict: Optional[dict] = None,
                                        make_sequence_length_divisible_by: int = 1):
    """Return ``(BatchedDataDict of [B, S] tensors, input_lengths [B])``."""
    pad_value_dict = pad_value_dict or {}
    flats = [message_log_to_flat(log) for log in message_logs]
    lengths = torch.tensor([f["token_ids"].shape[0] if "token_ids" in f else 0 for f in flats], dtype=torch.int64)
    S = int(lengths.max()) if len(lengths) else 0
    m = max(1, make_sequence_length_divisible_by)
    S = (S + m - 1) // m * m
    keys = sorted({k for f in flats for k in f})
    out = BatchedDataDict()
    for k in keys:
        ref = next(f[k] for f in flats if k in f)
        t = torch.full((len(flats), S) + tuple(ref.shape[1:]), pad_value_dict.get(k, PAD_VALUES.get(k, 0)),
                       dtype=ref.dtype)
        for i, f in enumerate(flats):
            if k in f:
                t[i, : f[k].shape[0]] = f[k]
        out[k] = t
    return out, lengths
