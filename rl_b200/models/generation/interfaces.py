"""Generation interface and data contracts.

Mirrors the reference's ``GenerationInterface`` (``nemo_rl/models/generation/interfaces.py:495``)
and its data specs: ``GenerationDatumSpec`` (``:350``; right-padded ``input_ids`` and
``input_lengths``) and ``GenerationOutputSpec`` (``:384``; ``output_ids`` = prompt +
generated tokens right-padded, ``logprobs`` aligned to token positions with 0
on prompt / padding positions, ``generation_lengths``,
``unpadded_sequence_lengths``, ``truncated``).
"""

from __future__ import annotations

from typing import Any, Optional, Protocol, TypedDict

import torch


class GenerationConfig(TypedDict, total=False):
    backend: str
    max_new_tokens: int
    temperature: float
    top_p: float
    top_k: Optional[int]
    stop_token_ids: Optional[list[int]]
    stop_strings: Optional[list[str]]
    pad_token_id: int
    colocated: dict
    kv_cache_dtype: str
    block_size_tokens: int
    use_cuda_graphs: bool
    max_num_seqs: int


class GenerationDatumSpec(TypedDict):
    input_ids: torch.Tensor
    input_lengths: torch.Tensor


class GenerationOutputSpec(TypedDict):
    output_ids: torch.Tensor
    logprobs: torch.Tensor
    generation_lengths: torch.Tensor
    unpadded_sequence_lengths: torch.Tensor
    truncated: torch.Tensor


class GenerationInterface(Protocol):
    def generate(self, data: Any, greedy: bool = False) -> Any: ...

    def prepare_for_generation(self, *args, **kwargs) -> bool: ...

    def finish_generation(self, *args, **kwargs) -> bool: ...

    def update_weights_from_training(self) -> None: ...

    def invalidate_kv_cache(self) -> bool: ...

    def shutdown(self) -> bool: ...
