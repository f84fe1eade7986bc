"""Mixture-of-experts token routing (K10-K12).

``moe_forward_local`` runs all experts on this rank: tokens are permuted into
expert-contiguous order (stable sort of the flattened top-k assignment), each
expert applies SwiGLU(x W13^T) W2^T to its segment, and results are combined
with the routing weights by an index-add.  This is the portable (CPU) path
and the numerics oracle of the fused CUDA path in :mod:`psrl_b200.ops.moe`.
"""

from __future__ import annotations

import torch

from .. import ops


def permute_by_expert(idx: torch.Tensor, num_experts: int):
    """For a [T, k] expert assignment return (order, token_of_row, counts)."""
    T, k = idx.shape
    flat = idx.reshape(-1)
    order = torch.argsort(flat, stable=True)
    token_of = order // k
    counts = torch.bincount(flat, minlength=num_experts)
    return order, token_of, counts


def grouped_swiglu_mlp(xs: torch.Tensor, counts: list[int], w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """Apply expert e's SwiGLU MLP to its contiguous segment of ``xs``."""
    out = torch.empty(xs.shape[0], w2.shape[1], dtype=xs.dtype, device=xs.device)
    start = 0
    for e, n in enumerate(counts):
        if n:
            seg = xs[start: start + n]
            out[start: start + n] = ops.swiglu(seg @ w13[e].t()) @ w2[e].t()
        start += n
    return out


def moe_forward_local(x: torch.Tensor, w: torch.Tensor, idx: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor):
    T, h = x.shape
    E = w13.shape[0]
    order, token_of, counts = permute_by_expert(idx, E)
    xs = x[token_of]
    ys = grouped_swiglu_mlp(xs, counts.tolist(), w13, w2)
    wts = w.reshape(-1)[order].to(ys.dtype)
    y = torch.zeros(T, h, dtype=torch.float32, device=x.device)
    y.index_add_(0, token_of, (ys * wts[:, None]).float())
    return y.to(x.dtype)
