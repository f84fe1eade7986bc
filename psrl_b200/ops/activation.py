"""SwiGLU activation (K7) on a fused [gate | up] projection.  CUDA: ``csrc/elementwise.cu``."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext


def swiglu_ref(gu: torch.Tensor) -> torch.Tensor:
    g, u = gu.chunk(2, dim=-1)
    return (F.silu(g.float()) * u.float()).to(gu.dtype)


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ctx.save_for_backward(gu)
        return ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dout):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(gu, dout.contiguous())


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    if gu.is_cuda and gu.dtype == torch.bfloat16:
        return _SwiGLUFn.apply(gu)
    return swiglu_ref(gu)
