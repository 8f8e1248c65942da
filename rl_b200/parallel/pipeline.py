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

Pairing (why the executor batches): NCCL runs the point-to-point work between
two ranks on one stream per communicator, in posting order, and a send larger
than its channel buffer completes only together with the peer's matching
receive.  At two stages, 1F1B has rank 0 send ``f1`` and then receive ``g0``
while rank 1 sends ``g0`` and then receives ``f1``: as four separate
operations each rank's stream holds a send its peer answers only after its own
send, a cyclic wait.  The executor therefore posts the send of one plan step
and the receive of the next step in ONE ``batch_isend_irecv`` call whenever
both go to the same peer (an NCCL group: the two make progress together), and
separately otherwise; this is the pairing of Megatron's
``send_forward_recv_backward`` / ``send_backward_recv_forward``.
``simulate_rendezvous`` checks the plans against exactly this behaviour.

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
    ordered by stage) on the pipeline group."""

    def __init__(self, ps):
        self.ps = ps
        self.stage, self.n = ps.pp_rank, ps.pp_size
        self.group = ps.pp_group
        self.ranks = list(ps.pp_ranks)
        self.me = self.ranks[self.stage]
        self.prev = ps.pp_ranks[self.stage - 1] if self.stage > 0 else None
        self.next = ps.pp_ranks[self.stage + 1] if self.stage + 1 < self.n else None
        self._pending: list = []  # (work, tensor kept alive until the send completed)

    def exchange(self, send: Optional[tuple], recv: Optional[tuple]) -> Optional[torch.Tensor]:
        """Post ``send = (tensor, dst_stage)`` and ``recv = (shape, dtype, device,
        src_stage)`` (either may be None); returns the received tensor once it
        arrived (stream-ordered).  A send and a receive with the same peer are
        posted together as one group; otherwise the send is posted first and left
        in flight (``wait`` completes it)."""
        ops, buf = [], None
        if send is not None:
            t = send[0].contiguous()
            ops.append(dist.P2POp(dist.isend, t, self.ranks[send[1]], group=self.group))
        if recv is not None:
            shape, dtype, device, src = recv
            buf = torch.empty(shape, dtype=dtype, device=device)
            rop = dist.P2POp(dist.irecv, buf, self.ranks[src], group=self.group)
        if send is not None and recv is not None and send[1] == recv[3]:
            for w in dist.batch_isend_irecv(ops + [rop]):
                w.wait()
            return buf
        if send is not None:
            self._pending.append((dist.batch_isend_irecv(ops)[0], ops[0].tensor))
        if recv is not None:
            dist.batch_isend_irecv([rop])[0].wait()
        return buf

    def send_to_stage(self, t: torch.Tensor, stage: int) -> None:
        self.exchange((t, stage), None)

    def recv_from_stage(self, shape, dtype, device, stage: int) -> torch.Tensor:
        return self.exchange(None, (shape, dtype, device, stage))

    def send_forward(self, t: torch.Tensor) -> None:
        self.send_to_stage(t, self.stage + 1)

    def recv_forward(self, shape, dtype, device) -> torch.Tensor:
        return self.recv_from_stage(shape, dtype, device, self.stage - 1)

    def send_backward(self, g: torch.Tensor) -> None:
        self.send_to_stage(g, self.stage - 1)

    def recv_backward(self, shape, dtype, device) -> torch.Tensor:
        return self.recv_from_stage(shape, dtype, device, self.stage + 1)

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
    chunk ``v + 1``.  Micro-batches go in rounds of ``S`` (Megatron's
    interleaving unit): each round runs its forwards chunk by chunk; after all
    forwards, each round runs its backwards in reverse chunk order.  Rounds bound
    the messages in flight on the wrap-around edge to one round, which keeps the
    paired point-to-point posting free of cyclic waits (see
    ``simulate_rendezvous``)."""
    S, s, V, M = num_stages, stage, num_chunks, num_microbatches
    rounds = [range(g, min(g + S, M)) for g in range(0, M, S)]
    out = []
    for mbs in rounds:
        for v in range(V):
            first, last = s == 0 and v == 0, s == S - 1 and v == V - 1
            for i in mbs:
                out.append(PlanStep("F", v, i, None if first else (s - 1) % S, None if last else (s + 1) % S))
    if backward:
        for mbs in rounds:
            for v in reversed(range(V)):
                first, last = s == 0 and v == 0, s == S - 1 and v == V - 1
                for i in mbs:
                    out.append(PlanStep("B", v, i, None if last else (s + 1) % S, None if first else (s - 1) % S))
    return out


def _run_plan(comm: PipelineComm, plan: list[PlanStep],
              forward: Callable[[int, int, Optional[torch.Tensor]], torch.Tensor],
              in_shape: Callable[[int], tuple], dtype: torch.dtype, device: torch.device, backward: bool) -> None:
    """Execute a plan: the receive of step k + 1 is posted together with the send
    of step k (one group when they share a peer, see the module docstring)."""
    live: dict = {}

    def recv_spec(st: PlanStep):
        if st.recv_from is None:
            return None
        if st.kind == "F":
            return (in_shape(st.mb), dtype, device, st.recv_from)
        out = live[(st.chunk, st.mb)][1]
        return (out.shape, out.dtype, device, st.recv_from)

    got = comm.exchange(None, recv_spec(plan[0])) if plan else None
    for k, st in enumerate(plan):
        send = None
        if st.kind == "F":
            inp = got
            if inp is not None and backward:
                inp.requires_grad_(True)
            out = forward(st.mb, st.chunk, inp)
            if st.send_to is not None:
                send = (out.detach(), st.send_to)
            if backward:
                live[(st.chunk, st.mb)] = (inp, out)
        else:
            inp, out = live.pop((st.chunk, st.mb))
            if st.recv_from is None:
                out.backward()
            else:
                torch.autograd.backward(out, got)
            if st.send_to is not None:
                send = (inp.grad, st.send_to)
            del inp, out
        nxt = recv_spec(plan[k + 1]) if k + 1 < len(plan) else None
        got = comm.exchange(send, nxt) if (send is not None or nxt is not None) else None
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


def simulate_rendezvous(plans: list[list[PlanStep]], pair_same_peer: bool = True) -> bool:
    """Whether the per-rank plans finish under NCCL's worst case for large
    messages, executed as :func:`_run_plan` posts them: one communicator stream
    per rank pair running its operations in posting order; a send and its
    receive complete only together (neither side buffers); an operation posted
    after step k's compute starts only once that compute finished (the stream
    waits for the compute stream at posting); the receive of step k + 1 is
    posted with the send of step k, as one group when they share a peer
    (``pair_same_peer``; False posts them separately, send first).  A grouped
    receive releases its compute only when the whole group finished.  Returns
    False on a deadlock."""
    S = len(plans)

    def msg_of(r, st, sending):
        # a forward's output is the next virtual stage's input; a backward's input
        # gradient is the previous virtual stage's output gradient
        if sending:
            ch = st.chunk + (1 if st.kind == "F" and st.send_to == 0 and r == S - 1 else 0) \
                - (1 if st.kind == "B" and st.send_to == S - 1 and r == 0 else 0)
            return (st.kind, ch, st.mb, r, st.send_to)
        return (st.kind, st.chunk, st.mb, st.recv_from, r)

    streams = [dict() for _ in range(S)]  # rank -> peer -> list of items (each a list of ops)
    computes = []
    for r, plan in enumerate(plans):
        comps = [{"done": False, "wait": None} for _ in plan]
        computes.append(comps)

        def post(items_ops, after):
            for ops in items_ops:
                item = {"ops": ops, "after": after}
                for op in ops:
                    op["item"] = item
                streams[r].setdefault(ops[0]["peer"], []).append(item)

        def recv_op(k):
            st = plan[k]
            if st.recv_from is None:
                return None
            return {"kind": "recv", "msg": msg_of(r, st, False), "peer": st.recv_from, "done": False}

        first = recv_op(0) if plan else None
        if first is not None:
            post([[first]], None)
            comps[0]["wait"] = first
        for k, st in enumerate(plan):
            send = None
            if st.send_to is not None:
                send = {"kind": "send", "msg": msg_of(r, st, True), "peer": st.send_to, "done": False}
            rv = recv_op(k + 1) if k + 1 < len(plan) else None
            if send is not None and rv is not None and pair_same_peer and send["peer"] == rv["peer"]:
                post([[send, rv]], comps[k])
                comps[k + 1]["wait"] = ("group", send, rv)
            else:
                post([[x] for x in (send, rv) if x is not None], comps[k])
                if rv is not None:
                    comps[k + 1]["wait"] = rv

    def head(r, peer):
        for item in streams[r].get(peer, []):
            if not all(op["done"] for op in item["ops"]):
                return item
        return None

    def active(item):
        return item is not None and (item["after"] is None or item["after"]["done"])

    progress = True
    while progress:
        progress = False
        for r in range(S):
            for c in computes[r]:
                if c["done"]:
                    continue
                w = c["wait"]
                ok = w is None or (all(x["done"] for x in w[1:]) if isinstance(w, tuple) else w["done"])
                if ok:
                    c["done"] = True
                    progress = True
                break
        for r in range(S):
            for peer in list(streams[r]):
                it = head(r, peer)
                if not active(it):
                    continue
                pit = head(peer, r)
                if not active(pit):
                    continue
                for op in it["ops"]:
                    if op["done"] or op["kind"] != "send":
                        continue
                    for pop in pit["ops"]:
                        if not pop["done"] and pop["kind"] == "recv" and pop["msg"] == op["msg"]:
                            op["done"] = pop["done"] = True
                            progress = True
    return all(c["done"] for cs in computes for c in cs) and \
        all(op["done"] for st in streams for q in st.values() for it in q for op in it["ops"])
