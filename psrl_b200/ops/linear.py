"""Projection GEMMs on the paired-CTA tcgen05 kernel (``csrc/gemm_2sm.cu``).

* :func:`matmul_nt` — ``C = A B^T`` for any mix of K-major / MN-major stored
  operands (bf16 out, or accumulated into an fp32 buffer with split-K).
* :func:`linear` — ``x W^T (+ b)`` with autograd: forward, data gradient
  (``dy W``: B read MN-major straight from the weight) and weight gradient
  (``dy^T x``: both operands read MN-major straight from the activations)
  are all the same kernel, so no transposed copy is ever made.
* :func:`gate_up_swiglu` — the MLP's gate_up projection with SwiGLU fused
  into the GEMM epilogue; returns ``h = silu(gate) * up`` and keeps
  ``gate_up`` for the backward.

The reference runs these projections through cuBLAS under veRL / vLLM
(``scripts/install_basic.sh:104``); here they are hand-written tcgen05 code.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ._ext import ext
from .gemm import _err

# raster group (tile rows visited together) and the resident pairs the split-K
# heuristic aims to fill
GROUP_M = 8
_PAIRS = 74


def supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Shapes the paired kernel takes: bf16 CUDA, 2-D, rows 16-byte aligned."""
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
            and w.dim() == 2 and x.shape[1] == w.shape[1] and x.shape[1] % 8 == 0 and w.shape[0] % 8 == 0
            and x.stride(1) == 1 and w.stride(1) == 1 and x.stride(0) % 8 == 0 and w.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0)


def matmul_nt(a: torch.Tensor, b: torch.Tensor, a_mn: bool = False, b_mn: bool = False,
              out: torch.Tensor | None = None, splits: int = 1, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``A B^T``; ``a`` is stored [M, K] (or [K, M] with ``a_mn``), ``b`` [N, K]
    (or [K, N] with ``b_mn``).  With ``out`` (fp32 [M, N]) the product is added
    into it, the K loop split ``splits`` ways."""
    return ext().tc_gemm2(a, b, bool(a_mn), bool(b_mn), out, int(splits), GROUP_M, bias, _err(a.device))


def _wgrad_splits(n: int, k: int, m: int) -> int:
    """K-splits for a weight gradient with output [n, k] reduced over m rows:
    enough work units for two waves of the resident pairs."""
    tiles = -(-n // 256) * -(-k // 256)
    if tiles >= 2 * _PAIRS:
        return 1
    return max(1, min(-(-2 * _PAIRS // tiles), m // 1024))


def weight_grad(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """``dy^T x`` ([N, K] bf16) for dy [M, N], x [M, K], read in place."""
    n, k, m = dy.shape[1], x.shape[1], dy.shape[0]
    splits = _wgrad_splits(n, k, m)
    if splits == 1:
        return matmul_nt(dy, x, a_mn=True, b_mn=True)
    acc = torch.zeros(n, k, dtype=torch.float32, device=dy.device)
    matmul_nt(dy, x, a_mn=True, b_mn=True, out=acc, splits=splits)
    return acc.to(torch.bfloat16)


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.has_bias = b is not None
        return matmul_nt(x, w, bias=b)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = matmul_nt(dy, w, b_mn=True) if ctx.needs_input_grad[0] else None
        dw = weight_grad(dy, x) if ctx.needs_input_grad[1] else None
        db = dy.float().sum(0).to(dy.dtype) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """``x W^T + b`` over the last dimension of ``x``; tcgen05 on CUDA bf16."""
    shp = x.shape
    x2 = x.reshape(-1, shp[-1])
    if x2.is_cuda and x2.dtype == torch.bfloat16:
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if not supported(x2, w):
            raise RuntimeError(f"tcgen05 linear: unsupported operands x{tuple(x2.shape)} w{tuple(w.shape)}")
        y = _LinearFn.apply(x2, w, b)
        return y.reshape(*shp[:-1], w.shape[0])
    return F.linear(x, w, b)


class _GateUpSwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        gu, h = ext().tc_gemm2_swiglu(x, w, GROUP_M, _err(x.device))
        ctx.save_for_backward(x, w, gu)
        return h

    @staticmethod
    def backward(ctx, dh):
        x, w, gu = ctx.saved_tensors
        dgu = ext().swiglu_bwd(gu, dh.contiguous())
        dx = matmul_nt(dgu, w, b_mn=True) if ctx.needs_input_grad[0] else None
        dw = weight_grad(dgu, x) if ctx.needs_input_grad[1] else None
        return dx, dw


def gate_up_swiglu(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``silu(x Wg^T) * (x Wu^T)`` for the fused ``w = [Wg; Wu]``."""
    if x.is_cuda and x.dtype == torch.bfloat16:
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        if not supported(x2, w):
            raise RuntimeError(f"tcgen05 gate_up: unsupported operands x{tuple(x2.shape)} w{tuple(w.shape)}")
        if (w.shape[0] // 2) % 128:
            # the fused epilogue pairs 128-row gate and up blocks; other widths
            # run the projection and the activation as two kernels
            from .activation import swiglu
            return swiglu(linear(x2, w)).reshape(*x.shape[:-1], w.shape[0] // 2)
        return _GateUpSwiGLUFn.apply(x2, w).reshape(*x.shape[:-1], w.shape[0] // 2)
    from .activation import swiglu_ref
    return swiglu_ref(F.linear(x, w))


# ------------------------------------------------------------------- decode
def _skinny(x, w, b, swiglu: bool, split: int) -> torch.Tensor:
    B = x.shape[0]
    if B <= 256:
        return ext().tc_gemm_skinny(x, w, b, swiglu, int(split), _err(x.device))
    return torch.cat([ext().tc_gemm_skinny(x[i:i + 256], w, b, swiglu, int(split), _err(x.device))
                      for i in range(0, B, 256)], 0)


def decode_linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None, split: int = 0) -> torch.Tensor:
    """``x W^T + b`` for a decode step's ``x`` ([B, K], one row per sequence),
    one launch of the weight-streaming tcgen05 kernel per 256 rows
    (``csrc/gemm_skinny.cu``): the weight fills the MMA's M dimension, and when
    the 128-row tiles do not fill the GPU a cluster of ``split`` CTAs (1, 2, 4
    or 8; 0 = chosen from the shape) shares each tile's K loop and reduces the
    partial tiles through distributed shared memory."""
    return _skinny(x.contiguous(), w, b, False, split)


def decode_gate_up_swiglu(x: torch.Tensor, w: torch.Tensor, split: int = 0) -> torch.Tensor:
    """``silu(x W_gate^T) * (x W_up^T)`` for a decode step, with ``w`` the fused
    [2I, K] gate_up weight (gate rows first): one launch whose epilogue applies
    the activation, so the [B, 2I] projection never reaches HBM."""
    if (w.shape[0] // 2) % 128:
        from .activation import swiglu
        return swiglu(_skinny(x.contiguous(), w, None, False, split))
    return _skinny(x.contiguous(), w, None, True, split)
