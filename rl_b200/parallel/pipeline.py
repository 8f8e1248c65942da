"""Pipeline parallelism: point-to-point activation / gradient exchange and the
1F1B micro-batch schedule.

Each pipeline stage holds a contiguous range of decoder layers (the first also
the embedding, the last the final norm and the head; see
``rl_b200.models.transformer.stage_layers``).  A training step runs the
one-forward-one-backward schedule: stage ``s`` of ``S`` first runs
``min(S - s - 1, M)`` forwards, then alternates forward / backward until every
micro-batch went forward, then drains the remaining backwards.  Sends are
non-blocking and receives blocking; every stage's action list is a
topological order of the schedule's dependency graph, so no stage waits on a
send that comes later in another stage's list.  At most ``S - s`` micro-batches'
activations are alive on stage ``s`` (GPipe keeps all ``M``).

Activations cross NVLink by NCCL send / recv between the adjacent stages (the
same tensor-parallel rank of both), ``[T_local, H]`` in the compute dtype;
shapes are derived on both sides from the packing plan, so no shape message
precedes a tensor.

Reference: the Megatron-core pipeline schedule the reference's Megatron
policy worker calls (``get_forward_backward_func``,
``nemo_rl/models/megatron/train.py:572``) and its
``pipeline_model_parallel_size`` setting (``nemo_rl/models/megatron/setup.py:1304``).
"""

from __future__ import annotations

from collections import deque
from typing import Callable, Optional

import torch
import torch.distributed as dist

__all__ = ["PipelineComm", "one_f_one_b", "schedule_1f1b", "virtual_pipeline"]


class PipelineComm:
    """Send / receive between adjacent pipeline stages (global ranks from
    ``ps.pp_ranks``, ordered by stage)."""

    def __init__(self, ps):
        self.ps = ps
        self.stage, self.n = ps.pp_rank, ps.pp_size
        self.group = ps.pp_group
        self.prev = ps.pp_ranks[self.stage - 1] if self.stage > 0 else None
        self.next = ps.pp_ranks[self.stage + 1] if self.stage + 1 < self.n else None
        # virtual pipeline: chunk v of the last rank feeds chunk v + 1 of the first
        self.prev_wrap = ps.pp_ranks[(self.stage - 1) % self.n]
        self.next_wrap = ps.pp_ranks[(self.stage + 1) % self.n]
        self._pending: list = []  # (work, tensor kept alive until the send completed)

    def _send(self, t: torch.Tensor, dst: int) -> None:
        t = t.contiguous()
        self._pending.append((dist.isend(t, dst, group=self.group), t))

    def _recv(self, shape, dtype, device, src: int) -> torch.Tensor:
        buf = torch.empty(shape, dtype=dtype, device=device)
        dist.recv(buf, src, group=self.group)
        return buf

    def send_forward(self, t: torch.Tensor) -> None:
        self._send(t, self.next)

    def recv_forward(self, shape, dtype, device) -> torch.Tensor:
        return self._recv(shape, dtype, device, self.prev)

    def send_backward(self, g: torch.Tensor) -> None:
        self._send(g, self.prev)

    def recv_backward(self, shape, dtype, device) -> torch.Tensor:
        return self._recv(shape, dtype, device, self.next)

    def wait(self) -> None:
        for w, _ in self._pending:
            w.wait()
        self._pending.clear()


def schedule_1f1b(num_stages: int, stage: int, num_microbatches: int) -> list[tuple[str, int]]:
    """Action list of one stage: ("F", i) / ("B", i) in execution order."""
    M = num_microbatches
    warm = min(num_stages - stage - 1, M)
    acts: list[tuple[str, int]] = [("F", i) for i in range(warm)]
    f, b = warm, 0
    while f < M:
        acts.append(("F", f))
        f += 1
        acts.append(("B", b))
        b += 1
    while b < M:
        acts.append(("B", b))
        b += 1
    return acts


def one_f_one_b(comm: PipelineComm, num_microbatches: int, forward: Callable[[int, Optional[torch.Tensor]], torch.Tensor],
                in_shape: Callable[[int], tuple], dtype: torch.dtype, device: torch.device,
                backward: bool = True) -> None:
    """Run one training step's micro-batches through this stage.

    ``forward(i, hidden_in)`` runs micro-batch ``i`` on this stage: it returns
    the stage output ``[T_local, H]`` (non-last stages) or the scalar loss
    (last stage).  ``in_shape(i)`` is the shape of micro-batch ``i``'s stage
    input / output activation.  ``backward=False`` (evaluation) runs forwards
    only."""
    first, last = comm.stage == 0, comm.stage == comm.n - 1
    live: deque = deque()
    acts = schedule_1f1b(comm.n, comm.stage, num_microbatches) if backward else \
        [("F", i) for i in range(num_microbatches)]
    for kind, i in acts:
        if kind == "F":
            inp = None
            if not first:
                inp = comm.recv_forward(in_shape(i), dtype, device)
                if backward:
                    inp.requires_grad_(True)
            out = forward(i, inp)
            if not last:
                comm.send_forward(out.detach())
            if backward:
                live.append((inp, out))
        else:
            inp, out = live.popleft()
            if last:
                out.backward()
            else:
                g = comm.recv_backward(out.shape, out.dtype, device)
                torch.autograd.backward(out, g)
            if not first:
                comm.send_backward(inp.grad)
            del inp, out
    comm.wait()


def virtual_pipeline(comm: PipelineComm, num_microbatches: int, num_chunks: int,
                     forward: Callable[[int, int, Optional[torch.Tensor]], torch.Tensor],
                     in_shape: Callable[[int], tuple], dtype: torch.dtype, device: torch.device,
                     backward: bool = True) -> None:
    """Micro-batches through ``num_chunks`` model chunks per rank (virtual
    stage ``v * S + s`` is chunk ``v`` of rank ``s``; the last rank's chunk
    ``v`` feeds the first rank's chunk ``v + 1``).  Every rank runs all
    forwards chunk by chunk, then all backwards in reverse chunk order: each
    rank's order is a topological order of the virtual stages' dependencies and
    every rank pair exchanges messages in the order both sides expect, so the
    blocking receives never wait on a later send.  ``forward(i, v, hidden_in)``
    returns chunk ``v``'s output (the scalar loss on the last virtual stage).

    Reference: Megatron's interleaved schedule behind
    ``virtual_pipeline_model_parallel_size``; this order keeps every
    micro-batch's activations until the backward phase (GPipe memory) in
    exchange for a schedule without per-step coordination."""
    S, s, V, M = comm.n, comm.stage, num_chunks, num_microbatches
    live: dict = {}
    for v in range(V):
        first, last = s == 0 and v == 0, s == S - 1 and v == V - 1
        for i in range(M):
            inp = None
            if not first:
                inp = torch.empty(in_shape(i), dtype=dtype, device=device)
                dist.recv(inp, comm.prev_wrap, group=comm.group)
                if backward:
                    inp.requires_grad_(True)
            out = forward(i, v, inp)
            if not last:
                comm._send(out.detach(), comm.next_wrap)
            if backward:
                live[(v, i)] = (inp, out)
    if backward:
        for v in reversed(range(V)):
            first, last = s == 0 and v == 0, s == S - 1 and v == V - 1
            for i in range(M):
                inp, out = live.pop((v, i))
                if last:
                    out.backward()
                else:
                    g = torch.empty(out.shape, dtype=out.dtype, device=device)
                    dist.recv(g, comm.next_wrap, group=comm.group)
                    torch.autograd.backward(out, g)
                if not first:
                    comm._send(inp.grad, comm.prev_wrap)
                del inp, out
    comm.wait()

