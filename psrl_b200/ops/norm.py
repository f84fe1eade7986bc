"""Fused residual-add + RMSNorm (K4).  CUDA: ``csrc/norm.cu``."""

from __future__ import annotations

import torch

from ._ext import ext


def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    s = x if residual is None else (x + residual)
    xf = s.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return y.to(x.dtype), (s if residual is not None else None)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        r2 = residual.reshape(-1, shape[-1]).contiguous() if residual is not None else None
        y, rout, rstd = ext().rmsnorm_fwd(x2, r2, w, eps)
        s = rout if residual is not None else x2
        ctx.save_for_backward(s, w, rstd)
        ctx.has_res = residual is not None
        ctx.shape = shape
        y = y.view(shape)
        if residual is not None:
            return y, rout.view(shape)
        return y, None

    @staticmethod
    def backward(ctx, dy, dres):
        s, w, rstd = ctx.saved_tensors
        h = ctx.shape[-1]
        dy2 = dy.reshape(-1, h).contiguous()
        dr2 = dres.reshape(-1, h).contiguous() if dres is not None else None
        ds, dw = ext().rmsnorm_bwd(dy2, s, w, rstd, dr2)
        ds = ds.view(ctx.shape)
        return ds, dw.to(w.dtype), (ds if ctx.has_res else None), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """Returns ``(norm(x + residual) * w, x + residual)`` (second is None without residual)."""
    if x.is_cuda and x.dtype == torch.bfloat16:
        return _RMSNormFn.apply(x, w, residual, eps)
    return rms_norm_ref(x, w, eps, residual)


def head_rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Per-head RMSNorm over the last dim (Qwen3 q_norm / k_norm)."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)
