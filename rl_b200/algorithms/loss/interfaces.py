"""Loss-function protocol (reference: ``nemo_rl/algorithms/loss/interfaces.py:23,53,62``)."""

from __future__ import annotations

import enum
from typing import Any, Protocol

import torch


class LossType(enum.Enum):
    TOKEN_LEVEL = "token_level"
    SEQUENCE_LEVEL = "sequence_level"


class LossInputType(enum.Enum):
    """What the training loop hands the loss: sampled-token log-probabilities
    (``LOGPROB``), raw logits (``LOGIT``, distillation) or critic values (``VALUE``)."""

    LOGPROB = "logprob"
    LOGIT = "logit"
    VALUE = "value"
    DRAFT = "draft"


class LossFunction(Protocol):
    loss_type: LossType
    input_type: LossInputType

    def __call__(self, next_token_logprobs: torch.Tensor, data: Any, global_valid_seqs: torch.Tensor,
                 global_valid_toks: torch.Tensor, **kwargs) -> tuple[torch.Tensor, dict]:
        ...
