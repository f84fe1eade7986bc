"""Ulysses sequence parallelism for the trainer: one packed micro-batch split
over ``P`` ranks along the tokens, attention computed head-parallel.

veRL's FSDP engine, on which the reference builds its trainer, exposes this as
``ulysses_sequence_parallel_size`` (the reference's own recipes leave it at 1
and use Megatron context parallelism instead, which :mod:`.cp` provides).

Layout: the micro-batch's ``T`` packed tokens are padded at the end to
``T_pad = P * ceil(T / P)`` and rank ``r`` keeps the contiguous rows
``[r T_pad / P, (r + 1) T_pad / P)``.  Everything but attention is
token-local.  Around attention one all-to-all turns the rank's rows of all
heads into all rows of its ``1 / P`` of the heads (query heads
``[r nq / P, ...)`` and the KV heads they read, ``[r nkv / P, ...)``), the
varlen kernel runs over the whole micro-batch's ``cu_seqlens`` for those
heads, and a second all-to-all returns this rank's rows of every head's
output, in head order, for the output projection.  Padding rows belong to no
sequence; their attention output is set to zero.  Both all-to-alls move the
same bytes as the activations themselves (no key / value all-gather), so
Ulysses needs ``P`` to divide the KV head count; context parallelism has no
such limit.

The all-to-alls are NCCL on GPU and gloo on CPU; each one's backward is the
opposite all-to-all.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import ops


@dataclass
class UlyssesPlan:
    group: object
    world: int
    rank: int
    cu: torch.Tensor        # the micro-batch's cu_seqlens (int32), padding rows after cu[-1]
    max_q: int              # longest sequence
    t_pad: int              # padded token count (a multiple of world)
    n_real: int             # real tokens (cu[-1])


def _a2a(x: torch.Tensor, group) -> torch.Tensor:
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x.contiguous(), group=group)
    return out


class _RowsToHeads(torch.autograd.Function):
    """[T_loc, P * C] (column block j destined for rank j) -> [P * T_loc, C]
    (the rows of every rank, in rank order, of this rank's column block)."""

    @staticmethod
    def forward(ctx, x, group, world):
        ctx.group, ctx.world = group, world
        t = x.shape[0]
        send = x.reshape(t, world, -1).transpose(0, 1).contiguous()        # [P, T_loc, C]
        return _a2a(send, group).reshape(world * t, -1)

    @staticmethod
    def backward(ctx, g):
        world = ctx.world
        t = g.shape[0] // world
        back = _a2a(g.reshape(world, t, -1), ctx.group)                    # [P, T_loc, C] from each rank
        return back.transpose(0, 1).reshape(t, -1), None, None


class _HeadsToRows(torch.autograd.Function):
    """Inverse of :class:`_RowsToHeads`: [P * T_loc, C] -> [T_loc, P * C]."""

    @staticmethod
    def forward(ctx, y, group, world):
        ctx.group, ctx.world = group, world
        t = y.shape[0] // world
        back = _a2a(y.reshape(world, t, -1), group)
        return back.transpose(0, 1).reshape(t, -1)

    @staticmethod
    def backward(ctx, g):
        world = ctx.world
        t = g.shape[0]
        send = g.reshape(t, world, -1).transpose(0, 1).contiguous()
        return _a2a(send, ctx.group).reshape(world * t, -1), None, None


def ulysses_attention(q: torch.Tensor, kv: torch.Tensor, plan: UlyssesPlan, nq: int, nkv: int,
                      d: int) -> torch.Tensor:
    """q [T_loc, nq d] and kv [T_loc, 2 nkv d] (k heads, then v heads) of this
    rank's rows -> attention output [T_loc, nq d] of the same rows."""
    P = plan.world
    if nq % P or nkv % P:
        raise ValueError(f"Ulysses over {P} ranks needs {nq} query / {nkv} KV heads divisible by {P}")
    t = q.shape[0]
    qh, kh = nq // P, nkv // P
    # column block j: rank j's query heads, then its key heads, then its value heads
    x = torch.cat([q.reshape(t, P, qh * d), kv[:, : nkv * d].reshape(t, P, kh * d),
                   kv[:, nkv * d:].reshape(t, P, kh * d)], dim=-1).reshape(t, -1)
    y = _RowsToHeads.apply(x, plan.group, P)                                  # [T_pad, (qh + 2 kh) d]
    o = ops.varlen_attention(y[: plan.n_real].contiguous(), plan.cu, plan.max_q, qh, kh, d)
    if plan.t_pad > plan.n_real:                                              # padding rows: zero output
        o = torch.cat([o, o.new_zeros(plan.t_pad - plan.n_real, o.shape[1])])
    return _HeadsToRows.apply(o, plan.group, P)


class UlyssesShard:
    """One packed micro-batch cut to this rank's contiguous rows; the same
    interface as :class:`.cp.CPShard` (``local``, ``positions``, ``plan``,
    ``full``)."""

    def __init__(self, cu_seqlens: torch.Tensor, group):
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        cu = [int(v) for v in cu_seqlens.tolist()]
        n = cu[-1]
        t_loc = -(-n // world)
        t_pad = t_loc * world
        dev = cu_seqlens.device
        pos = []
        for j in range(len(cu) - 1):
            pos.extend(range(cu[j + 1] - cu[j]))
        pos.extend([0] * (t_pad - n))
        self.lo, self.hi, self.n = rank * t_loc, (rank + 1) * t_loc, n
        self.pos = torch.tensor(pos[self.lo:self.hi], dtype=torch.int32, device=dev)
        max_q = max((cu[j + 1] - cu[j] for j in range(len(cu) - 1)), default=0)
        self.plan = UlyssesPlan(group, world, rank, cu_seqlens.to(torch.int32), max_q, t_pad, n)

    def local(self, t: torch.Tensor, pad=0) -> torch.Tensor:
        x = t[self.lo:min(self.hi, self.n)]
        need = (self.hi - self.lo) - x.shape[0]       # padding rows at the end of the last ranks
        if need > 0:
            x = torch.cat([x, torch.full((need,) + tuple(t.shape[1:]), pad, dtype=t.dtype, device=t.device)])
        return x

    def positions(self) -> torch.Tensor:
        return self.pos

    def full(self, x: torch.Tensor) -> torch.Tensor:
        """Per-token values of every rank back in micro-batch order (no gradient)."""
        world = self.plan.world
        out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.plan.group)
        return out[: self.n]
