"""Dataset sample contracts (reference: ``nemo_rl/data/interfaces.py:63`` ``DatumSpec``).

A *message log* is a list of messages ``{"role", "content", "token_ids"}``;
the token ids of every message are what the model sees, concatenated in order.
"""

from __future__ import annotations

from typing import Any, NotRequired, Optional, TypedDict

import torch


class Message(TypedDict, total=False):
    role: str
    content: str
    token_ids: torch.Tensor
    generation_logprobs: torch.Tensor


class DatumSpec(TypedDict, total=False):
    message_log: list[Message]
    length: int
    extra_env_info: Optional[dict[str, Any]]
    loss_multiplier: float
    idx: int
    task_name: str
    stop_strings: NotRequired[Optional[list[str]]]


TaskDataSpec = dict
