"""Expert-parallel MoE dispatch / combine with direct peer stores over NVLink.

Replaces the NCCL path of ``TransformerLM._moe_ep_experts`` (all-to-all with
variable splits, then a per-(expert, source) regroup): every routed
(token, choice) row is stored by ONE kernel (``csrc/ep_comm.cu``) straight into
its final row of the expert owner's receive buffer - already grouped by local
expert, then by source rank - so the owner runs its grouped expert GEMM on the
buffer contents with no permutation.  The owner learns each row's origin from
a 32-bit tag stored beside it (source rank << 24 | assignment index) and
returns the expert outputs with the same kernel into the source's per-
assignment buffer; the source applies the routing weights.

Row placement (computed on the device; one small all-gather of the per-expert
counts and one host read of the row totals per layer):

    dst rank d = expert // E_local,  local expert l = expert % E_local
    row = sum_{l' < l} total(d, l') + sum_{s < me} count(s, d, l) + rank of the
          assignment among this rank's assignments to the same expert

The backward passes reuse the two exchanges in the opposite directions
(gradients of the received rows go back to the sources, gradients of the
returned rows go forward to the owners).

Reference: MCore ``moe_token_dispatcher_type: alltoall`` / DeepEP / HybridEP
(``examples/configs/recipes/llm/performance/grpo-qwen3-30ba3b-4n8g.yaml:25-29``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from rl_b200.ops._ext import ext
from rl_b200.parallel.symm import SymmetricBuffer

__all__ = ["EPExchange", "EPPlan", "ep_dispatch", "ep_combine", "make_plan"]


class EPExchange:
    """One direction of the exchange: double-buffered symmetric receive rows,
    tags, data flags and acks, sized for ``cap`` rows of ``H`` bf16."""

    def __init__(self, group, cap: int, H: int):
        self.group = group
        self.n = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.cap = int(cap)
        self.H = int(H)
        self.buf = SymmetricBuffer(max(16, 2 * self.cap * self.H * 2), group)
        self.tag = SymmetricBuffer(max(16, 2 * self.cap * 4), group)
        self.flags = SymmetricBuffer(2 * self.n * 4, group)
        self.acks = SymmetricBuffer(2 * self.n * 4, group)
        self.counter = torch.zeros(4, dtype=torch.int32, device="cuda")
        self.epoch = 0

    def _ptrs(self):
        return self.buf.ptrs, self.tag.ptrs, self.flags.ptrs, self.acks.ptrs

    def scatter(self, src: torch.Tensor, src_row, dst_rank, dst_row, tags=None) -> None:
        self.epoch += 1
        b, t, f, a = self._ptrs()
        ext().ep_scatter(src.contiguous(), src_row, dst_rank, dst_row, tags, self.cap, b, t, f, a, self.me,
                         self.epoch, self.counter)

    def consume(self, rows: int, want_tags: bool = False):
        out = torch.empty((rows, self.H), dtype=torch.bfloat16, device="cuda")
        tg = torch.empty(rows, dtype=torch.int32, device="cuda") if want_tags else None
        b, t, f, a = self._ptrs()
        ext().ep_consume(out, tg, self.cap, b, t, f, a, self.me, self.epoch, self.counter)
        return out, tg

    def close(self) -> None:
        for x in (self.buf, self.tag, self.flags, self.acks):
            x.close()


class EPPlan:
    """Where every routed row goes (this rank's view of one MoE layer call)."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def make_plan(ids: torch.Tensor, n: int, me: int, experts_local: int, group, perm=None) -> EPPlan:
    """``perm``: (stable expert-grouped order, tokens per expert) from the router
    kernel, when it produced them."""
    T, k = ids.shape
    E = n * experts_local
    flat = ids.reshape(-1)
    if perm is not None:
        order, counts = perm[0], perm[1].to(torch.int32)
    else:
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=E).to(torch.int32)
    sorted_e = flat[order]
    all_counts = torch.empty(n * E, dtype=torch.int32, device=ids.device)
    dist.all_gather_into_tensor(all_counts, counts, group=group)
    C = all_counts.view(n, n, experts_local).long()          # [src, dst, local expert]
    tot = C.sum(0)                                            # [dst, local expert]
    excl_l = torch.cumsum(tot, 1) - tot
    excl_s = torch.cumsum(C, 0) - C
    base = (excl_l + excl_s[me]).reshape(-1)                  # [E] first row of (me -> expert)
    start = torch.cumsum(counts.long(), 0) - counts.long()
    rank_in = torch.arange(T * k, device=ids.device) - start[sorted_e]
    dst_rank = (sorted_e // experts_local).to(torch.int32)
    dst_row = (base[sorted_e] + rank_in).to(torch.int32)
    tags = ((me << 24) | order).to(torch.int32)
    recv_total = tot.sum(1)                                   # rows each rank receives
    send_total = C.sum(dim=(1, 2))                            # T*k of each rank
    r_me, r_max, tk_max = torch.stack([recv_total[me], recv_total.max(), send_total.max()]).tolist()
    return EPPlan(T=T, k=k, order=order, src_tok=(order // k).to(torch.int32), src_assign=order.to(torch.int32),
                  dst_rank=dst_rank, dst_row=dst_row, tags=tags, counts_local=tot[me].to(torch.int32),
                  R=int(r_me), R_max=int(r_max), TK_max=int(tk_max), ret_rank=None, ret_row=None)


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, plan, ex_d, ex_c):
        ex_d.scatter(h, plan.src_tok, plan.dst_rank, plan.dst_row, plan.tags)
        xr, tg = ex_d.consume(plan.R, want_tags=True)
        plan.ret_rank = (tg >> 24).to(torch.int32)
        plan.ret_row = (tg & 0xFFFFFF).to(torch.int32)
        ctx.plan, ctx.ex_c = plan, ex_c
        return xr

    @staticmethod
    def backward(ctx, d_xr):
        plan = ctx.plan
        ctx.ex_c.scatter(d_xr.contiguous(), None, plan.ret_rank, plan.ret_row)
        d_assign, _ = ctx.ex_c.consume(plan.T * plan.k)
        return d_assign.view(plan.T, plan.k, -1).sum(1), None, None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, plan, ex_d, ex_c):
        ex_c.scatter(y.contiguous(), None, plan.ret_rank, plan.ret_row)
        ret, _ = ex_c.consume(plan.T * plan.k)
        ctx.plan, ctx.ex_d = plan, ex_d
        return ret

    @staticmethod
    def backward(ctx, d_ret):
        plan = ctx.plan
        ctx.ex_d.scatter(d_ret.contiguous(), plan.src_assign, plan.dst_rank, plan.dst_row)
        d_y, _ = ctx.ex_d.consume(plan.R)
        return d_y, None, None, None


def ep_dispatch(h, plan, ex_d, ex_c) -> torch.Tensor:
    """[T, H] token rows -> [R, H] rows owned by this rank's experts (grouped by local expert)."""
    return _Dispatch.apply(h, plan, ex_d, ex_c)


def ep_combine(y, plan, ex_d, ex_c) -> torch.Tensor:
    """[R, H] expert outputs -> [T*k, H] rows in this rank's assignment order (token-major)."""
    return _Combine.apply(y, plan, ex_d, ex_c)
