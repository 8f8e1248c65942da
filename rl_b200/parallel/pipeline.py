"""Pipeline parallelism: point-to-point activation / gradient exchange and the
1F1B and interleaved (virtual) micro-batch schedules.

Each pipeline stage holds a contiguous range of decoder layers (the first also
the embedding, the last the final norm and the head; see
``rl_b200.models.transformer.stage_layers``).  A training step runs the
one-forward-one-backward schedule: stage ``s`` of ``S`` first runs
``min(S - s - 1, M)`` forwards, then alternates forward / backward until every
micro-batch went forward, then drains the remaining backwards.  At most
``S - s`` micro-batches' activations are alive on stage ``s`` (GPipe keeps all
``M``).

Every schedule is first written as a plan: per rank, an ordered list of steps
``(kind, chunk, micro-batch, receive-from, send-to)``.  The executor follows the
plan literally, so the plan is what the deadlock check in the tests verifies.

Activations cross NVLink by NCCL send / recv between adjacent stages (the same
tensor-parallel rank of both), ``[T_local, H]`` in the compute dtype; shapes are
derived on both sides from the packing plan, so no shape message precedes a
tensor.

Why one process group per DIRECTED edge: NCCL runs all point-to-point work of
one communicator on one stream, in posting order, and a send larger than its
channel buffer finishes only once the peer's matching receive runs.  If both
directions of a rank pair shared a communicator, rank 0 could queue
``send(f1)`` ahead of ``recv(g0)`` while rank 1 queues ``send(g0)`` ahead of
``recv(f1)`` (1F1B at two stages), or the virtual schedule could queue all of
chunk 0's sends ahead of the wrap-around receive: each is a cyclic wait.  With
a communicator per direction, the stream of edge ``a -> b`` carries only
``a``'s sends (on ``a``) and ``b``'s matching receives (on ``b``), in the same
order on both sides, so a send can wait only on its own receive, which in turn
waits only on work that precedes it in the schedule's dependency order.

Reference: the Megatron-core pipeline schedule the reference's Megatron
policy worker calls (``get_forward_backward_func``,
``nemo_rl/models/megatron/train.py:572``) and its
``pipeline_model_parallel_size`` / ``virtual_pipeline_model_parallel_size``
settings (``nemo_rl/models/megatron/setup.py:1304``).
"""

from __future__ import annotations

from collections import deque
from typing import Callable, NamedTuple, Optional

import torch
import torch.distributed as dist

__all__ = ["PipelineComm", "PlanStep", "one_f_one_b", "plan_1f1b", "plan_virtual", "schedule_1f1b",
           "simulate_rendezvous", "virtual_pipeline"]


class PlanStep(NamedTuple):
    """One compute action of a rank.  ``recv_from`` / ``send_to`` are pipeline
    STAGE indices (None when the step receives / sends nothing): the input of a
    forward (or the output-gradient of a backward) arrives from ``recv_from``
    before the compute, and the result leaves for ``send_to`` after it."""

    kind: str  # "F" or "B"
    chunk: int
    mb: int
    recv_from: Optional[int]
    send_to: Optional[int]


class PipelineComm:
    """Send / receive between pipeline stages (global ranks from ``ps.pp_ranks``,
    ordered by stage).  Traffic from rank ``a`` to rank ``b`` uses the process
    group of the directed edge ``(a, b)`` from ``ps.pp_edge_groups`` when it is
    there (one communicator, hence one stream, per direction)."""

    def __init__(self, ps):
        self.ps = ps
        self.stage, self.n = ps.pp_rank, ps.pp_size
        self.group = ps.pp_group
        self.ranks = list(ps.pp_ranks)
        self.me = self.ranks[self.stage]
        self.edges = dict(getattr(ps, "pp_edge_groups", None) or {})
        self.prev = ps.pp_ranks[self.stage - 1] if self.stage > 0 else None
        self.next = ps.pp_ranks[self.stage + 1] if self.stage + 1 < self.n else None
        # virtual pipeline: chunk v of the last rank feeds chunk v + 1 of the first
        self.prev_wrap = ps.pp_ranks[(self.stage - 1) % self.n]
        self.next_wrap = ps.pp_ranks[(self.stage + 1) % self.n]
        self._pending: list = []  # (work, tensor kept alive until the send completed)

    def _group(self, src: int, dst: int):
        return self.edges.get((src, dst), self.group)

    def _send(self, t: torch.Tensor, dst: int) -> None:
        t = t.contiguous()
        self._pending.append((dist.isend(t, dst, group=self._group(self.me, dst)), t))

    def _recv(self, shape, dtype, device, src: int) -> torch.Tensor:
        buf = torch.empty(shape, dtype=dtype, device=device)
        dist.recv(buf, src, group=self._group(src, self.me))
        return buf

    def send_to_stage(self, t: torch.Tensor, stage: int) -> None:
        self._send(t, self.ranks[stage])

    def recv_from_stage(self, shape, dtype, device, stage: int) -> torch.Tensor:
        return self._recv(shape, dtype, device, self.ranks[stage])

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


def plan_1f1b(num_stages: int, stage: int, num_microbatches: int, backward: bool = True) -> list[PlanStep]:
    """The 1F1B plan of one stage (forwards only when ``backward`` is False)."""
    S, s = num_stages, stage
    acts = schedule_1f1b(S, s, num_microbatches) if backward else [("F", i) for i in range(num_microbatches)]
    out = []
    for kind, i in acts:
        if kind == "F":
            out.append(PlanStep("F", 0, i, s - 1 if s > 0 else None, s + 1 if s + 1 < S else None))
        else:
            out.append(PlanStep("B", 0, i, s + 1 if s + 1 < S else None, s - 1 if s > 0 else None))
    return out


def plan_virtual(num_stages: int, stage: int, num_microbatches: int, num_chunks: int,
                 backward: bool = True) -> list[PlanStep]:
    """The interleaved plan of one rank: virtual stage ``v * S + s`` is chunk
    ``v`` of rank ``s``; the last rank's chunk ``v`` feeds the first rank's
    chunk ``v + 1``.  Every rank runs all forwards chunk by chunk, then all
    backwards in reverse chunk order, which is a topological order of the
    virtual stages' dependencies on every rank."""
    S, s, V, M = num_stages, stage, num_chunks, num_microbatches
    out = []
    for v in range(V):
        first, last = s == 0 and v == 0, s == S - 1 and v == V - 1
        for i in range(M):
            out.append(PlanStep("F", v, i, None if first else (s - 1) % S, None if last else (s + 1) % S))
    if backward:
        for v in reversed(range(V)):
            first, last = s == 0 and v == 0, s == S - 1 and v == V - 1
            for i in range(M):
                out.append(PlanStep("B", v, i, None if last else (s + 1) % S, None if first else (s - 1) % S))
    return out


def _run_plan(comm: PipelineComm, plan: list[PlanStep],
              forward: Callable[[int, int, Optional[torch.Tensor]], torch.Tensor],
              in_shape: Callable[[int], tuple], dtype: torch.dtype, device: torch.device, backward: bool) -> None:
    live: dict = {}
    order: deque = deque()
    for st in plan:
        if st.kind == "F":
            inp = None
            if st.recv_from is not None:
                inp = comm.recv_from_stage(in_shape(st.mb), dtype, device, st.recv_from)
                if backward:
                    inp.requires_grad_(True)
            out = forward(st.mb, st.chunk, inp)
            if st.send_to is not None:
                comm.send_to_stage(out.detach(), st.send_to)
            if backward:
                live[(st.chunk, st.mb)] = (inp, out)
                order.append((st.chunk, st.mb))
        else:
            inp, out = live.pop((st.chunk, st.mb))
            if st.recv_from is None:
                out.backward()
            else:
                g = comm.recv_from_stage(out.shape, out.dtype, device, st.recv_from)
                torch.autograd.backward(out, g)
            if st.send_to is not None:
                comm.send_to_stage(inp.grad, st.send_to)
            del inp, out
    comm.wait()


def one_f_one_b(comm: PipelineComm, num_microbatches: int, forward: Callable[[int, Optional[torch.Tensor]], torch.Tensor],
                in_shape: Callable[[int], tuple], dtype: torch.dtype, device: torch.device,
                backward: bool = True) -> None:
    """Run one training step's micro-batches through this stage.

    ``forward(i, hidden_in)`` runs micro-batch ``i`` on this stage: it returns
    the stage output ``[T_local, H]`` (non-last stages) or the scalar loss
    (last stage).  ``in_shape(i)`` is the shape of micro-batch ``i``'s stage
    input / output activation.  ``backward=False`` (evaluation) runs forwards
    only."""
    plan = plan_1f1b(comm.n, comm.stage, num_microbatches, backward)
    _run_plan(comm, plan, lambda i, v, h: forward(i, h), in_shape, dtype, device, backward)


def virtual_pipeline(comm: PipelineComm, num_microbatches: int, num_chunks: int,
                     forward: Callable[[int, int, Optional[torch.Tensor]], torch.Tensor],
                     in_shape: Callable[[int], tuple], dtype: torch.dtype, device: torch.device,
                     backward: bool = True) -> None:
    """Micro-batches through ``num_chunks`` model chunks per rank
    (:func:`plan_virtual`).  ``forward(i, v, hidden_in)`` returns chunk ``v``'s
    output (the scalar loss on the last virtual stage).  This order keeps every
    micro-batch's activations until the backward phase (GPipe memory) in
    exchange for a schedule without per-step coordination.

    Reference: Megatron's interleaved schedule behind
    ``virtual_pipeline_model_parallel_size``."""
    plan = plan_virtual(comm.n, comm.stage, num_microbatches, num_chunks, backward)
    _run_plan(comm, plan, forward, in_shape, dtype, device, backward)


def simulate_rendezvous(plans: list[list[PlanStep]], directed: bool = True) -> bool:
    """Whether the per-rank plans finish under NCCL's worst case for large
    messages: every communicator runs its point-to-point operations on one
    stream in posting order, and a send and its receive complete only together
    (neither side buffers).  ``directed`` gives each direction of a rank pair
    its own communicator (what :class:`PipelineComm` does); False shares one
    communicator per pair.  Each rank's compute stream runs its plan in order;
    a compute waits for its receive, a send for its compute.  Returns False on a
    deadlock (no operation can make progress before all are done)."""
    S = len(plans)
    # per rank: comm streams keyed by communicator; items are [op, done]
    streams: list[dict] = [dict() for _ in range(S)]
    compute: list[list] = []
    for r, plan in enumerate(plans):
        items = []
        for k, st in enumerate(plan):
            recv = send = None
            if st.recv_from is not None:
                key = (st.recv_from, r) if directed else frozenset((st.recv_from, r))
                msg = (st.kind, st.chunk, st.mb, st.recv_from, r)
                recv = {"kind": "recv", "msg": msg, "done": False}
                streams[r].setdefault(key, []).append(recv)
            comp = {"done": False, "recv": recv}
            items.append(comp)
            if st.send_to is not None:
                key = (r, st.send_to) if directed else frozenset((r, st.send_to))
                # a forward's output is the next virtual stage's forward input; a backward's
                # input gradient is the previous stage's backward output-gradient
                msg = (st.kind, st.chunk + (1 if st.kind == "F" and st.send_to == 0 and r == S - 1 else 0)
                       - (1 if st.kind == "B" and st.send_to == S - 1 and r == 0 else 0), st.mb, r, st.send_to)
                send = {"kind": "send", "msg": msg, "done": False, "after": comp}
                streams[r].setdefault(key, []).append(send)
        compute.append(items)

    def head(q):
        for op in q:
            if not op["done"]:
                return op
        return None

    progress = True
    while progress:
        progress = False
        for r in range(S):
            for comp in compute[r]:
                if comp["done"]:
                    continue
                if comp["recv"] is None or comp["recv"]["done"]:
                    comp["done"] = True
                    progress = True
                break
        # rendezvous: a send at the head of its stream whose data is ready meets the
        # receive at the head of the peer's stream for the same message
        for r in range(S):
            for key, q in streams[r].items():
                op = head(q)
                if op is None or op["kind"] != "send" or not op["after"]["done"]:
                    continue
                dst = op["msg"][4]
                pkey = key
                peer = head(streams[dst].get(pkey, []))
                if peer is not None and peer["kind"] == "recv" and peer["msg"] == op["msg"]:
                    op["done"] = peer["done"] = True
                    progress = True
    return all(c["done"] for items in compute for c in items) and \
        all(op["done"] for st in streams for q in st.values() for op in q)
