"""Environment protocol (reference: ``nemo_rl/environments/interfaces.py:26`` ``EnvironmentReturn``,
``:54`` ``EnvironmentInterface`` with ``step`` ``:56`` and ``global_post_process_and_metrics``).

Environments run in-process on the host (no actor hop): ``step`` receives the
batch of message logs and per-sample metadata and returns observations,
rewards and termination flags for every sample.
"""

from __future__ import annotations

from typing import Any, NamedTuple, Optional

import torch


class EnvironmentReturn(NamedTuple):
    observations: list[dict]
    metadata: list[Any]
    next_stop_strings: list[Optional[list[str]]]
    rewards: torch.Tensor
    terminateds: torch.Tensor
    answers: Optional[list[Optional[str]]] = None


class EnvironmentInterface:
    def step(self, message_log_batch: list[list[dict]], metadata: list[Any]) -> EnvironmentReturn:
        raise NotImplementedError

    def global_post_process_and_metrics(self, batch) -> tuple[Any, dict]:
        return batch, {}

    def shutdown(self) -> None:
        return None
