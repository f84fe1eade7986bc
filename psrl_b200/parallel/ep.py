"""Expert parallelism for the MoE trainer (K12 dispatch / combine).

With an expert-parallel group of size P, rank r holds experts
[r * E/P, (r + 1) * E/P) of every MoE layer (the router and everything else
stay replicated).  A layer's forward on rank r:

1. routes its own tokens (replicated router: softmax + prior, top-k);
2. sorts its (token, slot) pairs by global expert id, which also groups them
   by owning rank, and sends each rank its rows (``all_to_all_single`` with
   per-rank split sizes; the expert ids travel alongside);
3. runs its local experts on everything it received, grouped by local expert
   (the tcgen05 grouped GEMM on CUDA);
4. returns every row to its sender (the inverse all-to-all);
5. combines each token's k expert outputs with the routing weights.

Both all-to-alls are differentiable (the backward of one is the other), so
gradients reach the senders' tokens and each rank accumulates gradients only
for the experts it owns.  The collectives are NCCL on GPU (the baseline path)
and gloo on CPU.

Reference: Megatron expert parallelism as configured by the reference
(``psrl/utils/megatron_converter.py`` EP/ETP layouts; MoE recipe at EP=8).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class EPGroup:
    group: object
    world: int
    rank: int
    num_experts: int
    p2p: object = None       # parallel.ep_p2p.PeerAllToAll: dispatch / combine over NVLink peer memory

    @property
    def local(self) -> int:
        return self.num_experts // self.world

    @property
    def first(self) -> int:
        return self.rank * self.local


def make_ep_group(group, num_experts: int, device=None, p2p_bytes: int = 0) -> EPGroup:
    """``p2p_bytes`` > 0 on CUDA: dispatch and combine rows move through
    symmetric receive buffers of that size in peer memory (``ep_p2p``)
    instead of NCCL."""
    world = dist.get_world_size(group)
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} expert-parallel ranks")
    p2p = None
    if p2p_bytes > 0 and device is not None and torch.device(device).type == "cuda" and world > 1:
        from .ep_p2p import PeerAllToAll
        p2p = PeerAllToAll(group, device, int(p2p_bytes))
    return EPGroup(group, world, dist.get_rank(group), num_experts, p2p)


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, out_splits, in_splits, group):
        ctx.splits = (out_splits, in_splits)
        ctx.group = group
        out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out_splits, in_splits = ctx.splits
        gi = g.new_empty((sum(in_splits),) + tuple(g.shape[1:]))
        dist.all_to_all_single(gi, g.contiguous(), in_splits, out_splits, group=ctx.group)
        return gi, None, None, None


def all_to_all(x: torch.Tensor, out_splits: list[int], in_splits: list[int], group) -> torch.Tensor:
    return _AllToAll.apply(x, out_splits, in_splits, group)


def _local_experts(xs: torch.Tensor, local_ids: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """SwiGLU experts on rows already assigned to local experts (any order)."""
    from .. import ops
    E = w13.shape[0]
    order = torch.argsort(local_ids, stable=True)
    counts = torch.bincount(local_ids, minlength=E)
    xs_sorted = xs.index_select(0, order)
    from ..ops import moe as moe_ops
    if moe_ops.supported(xs_sorted, w13, w2) and xs_sorted.shape[0] > 0:
        seg = torch.zeros(E + 1, dtype=torch.int32, device=xs.device)
        seg[1:] = counts.cumsum(0).int()
        ys_sorted = moe_ops.grouped_linear(ops.swiglu(moe_ops.grouped_linear(xs_sorted, w13, seg)), w2, seg)
    else:
        from .moe import grouped_swiglu_mlp
        ys_sorted = grouped_swiglu_mlp(xs_sorted, counts.tolist(), w13, w2)
    return torch.zeros_like(ys_sorted).index_copy(0, order, ys_sorted)


def moe_forward_ep(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, w13_local: torch.Tensor,
                   w2_local: torch.Tensor, ep: EPGroup) -> torch.Tensor:
    """x [T, h], routing weights w [T, k] and global expert ids [T, k] of this
    rank's tokens; w13_local / w2_local: this rank's experts."""
    T, k = ids.shape
    flat = ids.reshape(-1).long()
    order = torch.argsort(flat, stable=True)            # by global expert id => by owner rank
    token_of = order // k
    dest = flat.index_select(0, order) // ep.local
    send = torch.bincount(dest, minlength=ep.world)
    xs = x.index_select(0, token_of)
    local_ids = (flat.index_select(0, order) - dest * ep.local).to(torch.int64)
    if ep.p2p is not None:
        # rows over NVLink peer memory; the count matrix (P x P ints) and the
        # expert ids (8 bytes a row) stay on NCCL
        from .ep_p2p import peer_all_to_all
        M = ep.p2p.counts(send.tolist())
        send_l, recv_l = list(M[ep.rank]), [M[s][ep.rank] for s in range(ep.world)]
        rx = peer_all_to_all(xs, M, ep.p2p)
    else:
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=ep.group)
        send_l, recv_l = send.tolist(), recv.tolist()
        rx = all_to_all(xs, recv_l, send_l, ep.group)
    rids = torch.empty(sum(recv_l), dtype=torch.int64, device=x.device)
    dist.all_to_all_single(rids, local_ids.contiguous(), recv_l, send_l, group=ep.group)
    ry = _local_experts(rx, rids, w13_local, w2_local)
    if ep.p2p is not None:
        back = peer_all_to_all(ry, [list(c) for c in zip(*M)], ep.p2p)
    else:
        back = all_to_all(ry, send_l, recv_l, ep.group)
    wts = w.reshape(-1).index_select(0, order).to(torch.float32)
    y = torch.zeros(T, x.shape[1], dtype=torch.float32, device=x.device)
    y = y.index_add(0, token_of, back.float() * wts[:, None])
    return y.to(x.dtype)


@torch.no_grad()
def shard_experts(model, ep: EPGroup) -> list[str]:
    """Keep only this rank's experts in every MoE layer of ``model`` (a full,
    deterministically initialised model); returns the expert parameter names."""
    names = []
    for i, layer in enumerate(model.layers):
        mlp = layer.mlp
        if not hasattr(mlp, "experts_w13"):
            continue
        sl = slice(ep.first, ep.first + ep.local)
        mlp.experts_w13 = torch.nn.Parameter(mlp.experts_w13.data[sl].clone())
        mlp.experts_w2 = torch.nn.Parameter(mlp.experts_w2.data[sl].clone())
        mlp.ep = ep
        names += [f"layers.{i}.mlp.experts_w13", f"layers.{i}.mlp.experts_w2"]
    return names
