"""Fused MoE routing and expert MLP ops (K10 router + top-k + permutation, K11
grouped expert GEMMs).

``moe_mlp(x, router_logits, prior, w13, w2, k, renorm)`` runs, on CUDA:

1. ``moe_route``   — softmax + prior, top-k, renormalisation, expert counts;
2. ``moe_permute`` — expert segment offsets and each (token, slot)'s row;
3. ``moe_gather``  — token rows into expert-sorted order;
4. ``tc_grouped_gemm`` with ``w13`` [E, 2I, h] — one persistent tcgen05 launch
   for all experts (tile schedule derived on the device, no host sync, so the
   decode path stays graph-capturable);
5. SwiGLU;
6. ``tc_grouped_gemm`` with ``w2`` [E, h, I];
7. ``moe_combine`` — weighted sum of each token's k expert outputs in fp32.

Gradients (training) flow through :class:`_GroupedLinearFn` (backward with
per-expert cuBLAS matmuls over the same segments) and through the combine
weights; the router's top-k selection is not differentiated, as in the
reference's routers.
"""

from __future__ import annotations

import torch

from ._ext import ext


def route_ref(logits: torch.Tensor, prior: torch.Tensor | None, k: int, renorm: bool):
    z = logits.float() + (prior.float() if prior is not None else 0.0)
    p = z.softmax(-1)
    w, ids = p.topk(k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w, ids.int()


def route(logits: torch.Tensor, prior: torch.Tensor | None, k: int, renorm: bool = True):
    """(weights fp32 [T, k], expert ids int32 [T, k], counts int32 [E])."""
    if logits.is_cuda:
        w, ids, counts = ext().moe_route(logits.float().contiguous(), prior, int(k), bool(renorm))
        return w, ids, counts
    w, ids = route_ref(logits, prior, k, renorm)
    counts = torch.bincount(ids.reshape(-1).long(), minlength=logits.shape[-1]).int()
    return w, ids, counts


class _GroupedLinearFn(torch.autograd.Function):
    """y[r] = x[r] @ w[e(r)]^T over expert segments (forward: tcgen05 grouped GEMM)."""

    @staticmethod
    def forward(ctx, x, w, seg, seg_host):
        err = torch.zeros(1, dtype=torch.int32, device=x.device)
        y = ext().tc_grouped_gemm(x.contiguous(), w.contiguous(), seg, err)
        ctx.save_for_backward(x, w)
        ctx.seg_host = seg_host
        ctx.err = err
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        seg = ctx.seg_host
        gx = torch.zeros_like(x)
        gw = torch.zeros_like(w)
        gy = gy.contiguous()
        for e in range(w.shape[0]):
            s, t = seg[e], seg[e + 1]
            if t > s:
                gx[s:t] = gy[s:t] @ w[e]
                gw[e] = gy[s:t].t() @ x[s:t]
        return gx, gw, None, None


def grouped_linear(x: torch.Tensor, w: torch.Tensor, seg: torch.Tensor) -> torch.Tensor:
    """x [R, K] expert-sorted rows, w [E, N, K], seg int32 [E+1] -> [R, N]."""
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        return _GroupedLinearFn.apply(x, w, seg, seg.tolist())
    err = torch.zeros(1, dtype=torch.int32, device=x.device)
    return ext().tc_grouped_gemm(x.contiguous(), w.contiguous(), seg, err)


class _GatherFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, token_of_row):
        ctx.save_for_backward(token_of_row)
        ctx.T = x.shape[0]
        return ext().moe_gather(x, token_of_row)

    @staticmethod
    def backward(ctx, g):
        (tor,) = ctx.saved_tensors
        gx = torch.zeros(ctx.T, g.shape[1], dtype=torch.float32, device=g.device)
        gx.index_add_(0, tor.long(), g.float())
        return gx.to(g.dtype), None


class _CombineFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ys, pos, w):
        ctx.save_for_backward(ys, pos, w)
        return ext().moe_combine(ys.contiguous(), pos, w.contiguous())

    @staticmethod
    def backward(ctx, gy):
        ys, pos, w = ctx.saved_tensors
        T, k = pos.shape
        p = pos.long()
        gys = torch.zeros_like(ys, dtype=torch.float32)
        gys.index_add_(0, p.reshape(-1), (gy.float()[:, None, :] * w[:, :, None]).reshape(T * k, -1))
        gw = (ys.float()[p] * gy.float()[:, None, :]).sum(-1)
        return gys.to(ys.dtype), None, gw


def supported(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> bool:
    """Shapes the fused CUDA path takes: bf16, K of both GEMMs a multiple of 64."""
    return (x.is_cuda and x.dtype == torch.bfloat16 and w13.dtype == torch.bfloat16 and x.shape[-1] % 64 == 0
            and w2.shape[-1] % 64 == 0 and w13.shape[0] <= 256)


def moe_mlp_routed(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, w13: torch.Tensor,
                   w2: torch.Tensor) -> torch.Tensor:
    """SwiGLU experts for a given routing (``w`` [T, k] combine weights, ``ids``
    [T, k] indices into ``w13`` / ``w2``), inference only.  The per-expert
    counts come from a device scatter-add, so nothing waits on the host."""
    from .activation import swiglu
    ids = ids.to(torch.int32).contiguous()
    counts = torch.zeros(w13.shape[0], dtype=torch.int32, device=x.device)
    counts.scatter_add_(0, ids.reshape(-1).long(), torch.ones(ids.numel(), dtype=torch.int32, device=x.device))
    pos, tor, seg, _ = ext().moe_permute(ids, counts, 128, 1)
    xs = _GatherFn.apply(x.contiguous(), tor)
    h = swiglu(grouped_linear(xs, w13, seg))
    ys = grouped_linear(h, w2, seg)
    return _CombineFn.apply(ys, pos, w.float())


def moe_mlp(x: torch.Tensor, router_logits: torch.Tensor, prior: torch.Tensor | None, w13: torch.Tensor,
            w2: torch.Tensor, k: int, renorm: bool = True) -> torch.Tensor:
    """Top-k routed SwiGLU experts on CUDA (see module docstring)."""
    from .activation import swiglu
    w, ids, counts = route(router_logits, prior, k, renorm)
    pos, tor, seg, _ = ext().moe_permute(ids, counts, 128, 1)
    xs = _GatherFn.apply(x.contiguous(), tor)
    h = swiglu(grouped_linear(xs, w13, seg))
    ys = grouped_linear(h, w2, seg)
    if torch.is_grad_enabled() and router_logits.requires_grad:
        # differentiate the combine weights through the (renormalised) softmax
        z = router_logits.float() + (prior.float() if prior is not None else 0.0)
        pk = z.softmax(-1).gather(-1, ids.long())
        w = pk / pk.sum(-1, keepdim=True) if renorm else pk
    return _CombineFn.apply(ys, pos, w)
