"""Context parallelism for the trainer: one packed micro-batch split over ``P``
ranks along the sequence (the reference gets it from Megatron's
context-parallel group, ``psrl/utils/config.py:119-126``).

Layout (zigzag, so causal work is balanced): every sequence of length ``L``
(a multiple of ``2P``) is cut into ``2P`` chunks of ``c = L / 2P`` tokens and
rank ``r`` keeps chunks ``r`` and ``2P - 1 - r``.  Everything but attention is
token-local, so a rank runs embeddings, norms, projections, MLPs and the
LM-head log-probs on its own ``L / P`` tokens of each sequence.  Attention:

* forward — each rank's keys and values (``2 nkv d`` columns, ~1 KB per token
  per layer for a 3B model) are all-gathered over the CP group and put back
  in sequence order; each local query chunk ``k`` then attends to the key
  prefix ``[0, (k + 1) c)`` of its sequence with the tcgen05 kernel for
  queries against separate keys (``ops.attention_kv``: the chunk's queries
  are the last ``c`` of those ``(k + 1) c`` positions);
* backward — autograd runs the kernel's backward, scatter-adds the prefix
  gradients into sequence order and reduce-scatters them back to the ranks
  that own the keys (NCCL reduce-scatter; all-reduce + slice on gloo).

Weight gradients are partial sums over a rank's tokens: reduce them over the
CP group (with the data-parallel reduction) like any data-parallel gradient.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops.attention import attention_kv


@dataclass
class CPPlan:
    """Index plan of one packed micro-batch on one CP rank."""

    world: int
    rank: int
    group: object
    local_idx: torch.Tensor      # [T / P] int64: full-batch row of each local row
    perm: torch.Tensor           # [T] int64: gathered row (rank-major) of each full-batch row
    kv_idx: torch.Tensor         # int64: full-batch key rows of every (sequence, local chunk) prefix
    cu_q: torch.Tensor           # int32 [E + 1]: local query rows of each entry
    cu_k: torch.Tensor           # int32 [E + 1]: rows of each entry's prefix in kv_idx
    max_q: int
    max_k: int
    local_seqlens: list          # tokens of each sequence on this rank

    @property
    def num_local(self) -> int:
        return int(self.local_idx.numel())

    def to(self, device) -> "CPPlan":
        mv = {k: getattr(self, k).to(device) for k in ("local_idx", "perm", "kv_idx", "cu_q", "cu_k")}
        return CPPlan(self.world, self.rank, self.group, max_q=self.max_q, max_k=self.max_k,
                      local_seqlens=self.local_seqlens, **mv)


def pad_lengths(seqlens: list[int], world: int) -> list[int]:
    """Sequence lengths rounded up to a multiple of ``2 * world``."""
    m = 2 * world
    return [-(-int(n) // m) * m for n in seqlens]


def zigzag_rows(seqlens: list[int], world: int, rank: int) -> list[int]:
    """Full-batch rows of ``rank``'s tokens, in local order (per sequence:
    chunk ``rank`` then chunk ``2 world - 1 - rank``)."""
    rows, start = [], 0
    for n in seqlens:
        if n % (2 * world):
            raise ValueError(f"sequence of {n} tokens does not split into {2 * world} equal chunks; pad it "
                             "(parallel.cp.pad_lengths)")
        c = n // (2 * world)
        for k in (rank, 2 * world - 1 - rank):
            rows.extend(range(start + k * c, start + (k + 1) * c))
        start += n
    return rows


def make_plan(seqlens: list[int], group=None, device="cpu") -> CPPlan:
    """Plan for a packed micro-batch of sequences with these lengths (each a
    multiple of ``2 P``) on this rank of the CP ``group``."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    all_rows = [zigzag_rows(seqlens, world, r) for r in range(world)]
    local = all_rows[rank]
    T = sum(seqlens)
    perm = torch.empty(T, dtype=torch.int64)
    flat = torch.tensor([i for rows in all_rows for i in rows], dtype=torch.int64)
    perm[flat] = torch.arange(T, dtype=torch.int64)
    kv_idx, cu_q, cu_k = [], [0], [0]
    start = 0
    for n in seqlens:
        c = n // (2 * world)
        for k in (rank, 2 * world - 1 - rank):
            kv_idx.extend(range(start, start + (k + 1) * c))
            cu_q.append(cu_q[-1] + c)
            cu_k.append(cu_k[-1] + (k + 1) * c)
        start += n
    n_ent = len(cu_q) - 1
    plan = CPPlan(world, rank, group, torch.tensor(local, dtype=torch.int64), perm,
                  torch.tensor(kv_idx, dtype=torch.int64), torch.tensor(cu_q, dtype=torch.int32),
                  torch.tensor(cu_k, dtype=torch.int32),
                  max_q=max((cu_q[i + 1] - cu_q[i] for i in range(n_ent)), default=0),
                  max_k=max((cu_k[i + 1] - cu_k[i] for i in range(n_ent)), default=0),
                  local_seqlens=[n // world for n in seqlens])
    return plan.to(device)


class _AllGatherRows(torch.autograd.Function):
    """[T_loc, C] per rank -> [P * T_loc, C] (rank-major); backward sums the
    gradient over ranks and returns this rank's rows."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        world = dist.get_world_size(group)
        out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        group = ctx.group
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        g = g.contiguous()
        n = g.shape[0] // world
        if dist.get_backend(group) == "nccl":
            out = torch.empty((n,) + tuple(g.shape[1:]), dtype=g.dtype, device=g.device)
            dist.reduce_scatter_tensor(out, g, group=group)
            return out, None
        dist.all_reduce(g, group=group)
        return g[rank * n:(rank + 1) * n].clone(), None


def cp_attention(q: torch.Tensor, kv: torch.Tensor, plan: CPPlan, nq: int, nkv: int, d: int,
                 scale: float | None = None) -> torch.Tensor:
    """Attention of this rank's queries ``q`` [T_loc, nq d] over the whole
    sequences, given this rank's keys / values ``kv`` [T_loc, 2 nkv d]."""
    full = _AllGatherRows.apply(kv, plan.group)[plan.perm]          # sequence order
    kv_pref = full.index_select(0, plan.kv_idx)                       # each chunk's key prefix
    return attention_kv(q, kv_pref, plan.cu_q, plan.cu_k, plan.max_q, plan.max_k, nq, nkv, d, scale)


def gather_tokens(x: torch.Tensor, plan: CPPlan) -> torch.Tensor:
    """Per-token values of every rank back in full-batch order (no gradient)."""
    world = plan.world
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=plan.group)
    return out[plan.perm]


class CPShard:
    """One packed micro-batch padded to CP-divisible sequence lengths and cut
    to this rank's zigzag share.  ``local(t, pad)`` cuts any per-token tensor
    of the micro-batch the same way (``pad`` fills the padding rows);
    ``full(x)`` gathers per-token results of every rank back into the
    micro-batch's original token order (padding dropped)."""

    def __init__(self, cu_seqlens: torch.Tensor, group):
        world = dist.get_world_size(group)
        cu = [int(v) for v in cu_seqlens.tolist()]
        lens = [cu[j + 1] - cu[j] for j in range(len(cu) - 1)]
        padded = pad_lengths(lens, world)
        dev = cu_seqlens.device
        src, pad_pos, real = [], [], []
        o = 0
        for j, (n, m) in enumerate(zip(lens, padded)):
            src.extend(range(cu[j], cu[j] + n))
            src.extend([-1] * (m - n))
            pad_pos.extend(range(m))
            real.extend(range(o, o + n))
            o += m
        self.src = torch.tensor(src, dtype=torch.int64, device=dev)          # padded row -> source row (-1: pad)
        self.pos = torch.tensor(pad_pos, dtype=torch.int32, device=dev)      # position within the sequence
        self.real = torch.tensor(real, dtype=torch.int64, device=dev)        # padded rows holding real tokens
        self.plan = make_plan(padded, group, dev)
        self._li = self.plan.local_idx
        self._lsrc = self.src[self._li]
        self._lpad = self._lsrc < 0

    def local(self, t: torch.Tensor, pad=0) -> torch.Tensor:
        x = t[self._lsrc.clamp(min=0)]
        if bool(self._lpad.any()):
            x = x.clone()
            x[self._lpad] = pad
        return x

    def positions(self) -> torch.Tensor:
        return self.pos[self._li]

    def full(self, x: torch.Tensor) -> torch.Tensor:
        return gather_tokens(x, self.plan)[self.real]
