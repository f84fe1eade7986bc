"""Tensor-parallel GEMMs fused with their all-reduce over NVLink (K15).

For a 2-rank tensor-parallel group, :class:`FusedTP` owns symmetric fp32
accumulators (two, used in turn) and a small flag array on every rank, maps
the peer's copies into this process (CUDA IPC over NVLink) and runs

    y = all_reduce(x @ W^T)         (row-parallel O / down projections)

as one tcgen05 GEMM whose epilogue adds each finished output tile into both
ranks' accumulators with TMA reduce-add (``csrc/gemm_2sm.cu``,
``tc_gemm2_allreduce2``), so the transfer over NVLink overlaps the tiles still
being computed; then a one-thread flag barrier (``csrc/tp_fused.cu``, bounded
wait with an error status) and a finalize kernel that converts the sum to bf16
and zeroes the accumulator for its next use.  With two accumulators used in
turn, one barrier per call orders every write into a peer's accumulator after
the peer has finished reading it.

The NCCL baseline is ``parallel/tp.py``'s all-reduce after a local GEMM; the
reference's layouts are Megatron's (``psrl/utils/converter/megatron_converter.py:526-560``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..ops.gemm import _err, check_errors
from ..ops.linear import GROUP_M, matmul_nt, weight_grad


class FusedTP:
    """Symmetric buffers and the fused row-parallel GEMM of one 2-rank group."""

    def __init__(self, group, device, max_elems: int, timeout_s: float = 2.0):
        self.group = group
        self.world = dist.get_world_size(group)
        if self.world != 2:
            raise ValueError("the fused tensor-parallel GEMM pairs exactly two ranks")
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.max_elems = int(max_elems)
        self.timeout_s = float(timeout_s)
        self.acc = [torch.zeros(self.max_elems, dtype=torch.float32, device=self.device) for _ in range(2)]
        self.flags = torch.zeros(64, dtype=torch.int32, device=self.device)   # slot r * 16 per rank
        mine = {"acc": [ops.ext().ipc_handle(a) for a in self.acc], "flags": ops.ext().ipc_handle(self.flags),
                "device": self.device.index}
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        peer = allh[1 - self.rank]
        if int(peer["device"]) != self.device.index:
            ops.ext().enable_peer_access(int(peer["device"]))
        self.peer_acc = [ops.ext().ipc_open(h, int(off), self.max_elems, torch.float32, int(peer["device"]))
                         for h, off in peer["acc"]]
        h, off = peer["flags"]
        peer_flags = ops.ext().ipc_open(h, int(off), 64, torch.int32, int(peer["device"]))
        # this rank writes its slot in both arrays; it reads both ranks' slots in its own
        slot = 16 * self.rank
        by_rank = {self.rank: self.flags, 1 - self.rank: peer_flags}
        self.slot_in = [by_rank[r][slot:slot + 1] for r in range(2)]
        self.own = [self.flags[16 * r:16 * r + 1] for r in range(2)]
        self.epoch = 0
        self.calls = 0

    def barrier(self) -> None:
        """Both ranks' previously launched kernels on their streams are complete
        and their writes visible (bounded wait; an expiry is reported by
        :func:`check_errors`)."""
        self.epoch += 1
        ops.ext().peer_barrier(self.slot_in, self.own, self.epoch, self.timeout_s, _err(self.device))

    def gemm_allreduce(self, x: torch.Tensor, w: torch.Tensor, b_mn: bool = False) -> torch.Tensor:
        """``all_reduce(x @ op(w)^T)`` over the pair: x [M, K] bf16; w [N, K]
        (or [K, N] with ``b_mn``, the data-gradient layout)."""
        M = x.shape[0]
        N = w.shape[1] if b_mn else w.shape[0]
        if M * N > self.max_elems:
            raise ValueError(f"fused all-reduce of {M}x{N} exceeds the {self.max_elems}-element accumulators")
        buf = self.calls & 1
        self.calls += 1
        acc = self.acc[buf][: M * N].view(M, N)
        peer = self.peer_acc[buf][: M * N].view(M, N)
        ops.ext().tc_gemm2_allreduce2(x.contiguous(), w, bool(b_mn), acc, peer, GROUP_M, _err(self.device))
        self.barrier()
        out = torch.empty(M, N, dtype=torch.bfloat16, device=self.device)
        ops.ext().acc_finalize(acc, out, None)
        return out

    def check(self) -> None:
        check_errors(self.device)


class _RowParallelFn(torch.autograd.Function):
    """y = all_reduce(x_local W_local^T); backward: dx_local = dy W_local (no
    communication), dW_local = dy^T x_local."""

    @staticmethod
    def forward(ctx, x, w, ftp):
        ctx.save_for_backward(x, w)
        return ftp.gemm_allreduce(x, w)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = matmul_nt(dy, w, b_mn=True) if ctx.needs_input_grad[0] else None
        dw = weight_grad(dy, x) if ctx.needs_input_grad[1] else None
        return dx, dw, None


class _ColumnParallelFn(torch.autograd.Function):
    """y_local = x W_local^T (no communication); backward: dx = all_reduce(dy_local
    W_local) in one fused kernel, dW_local = dy_local^T x."""

    @staticmethod
    def forward(ctx, x, w, b, ftp):
        ctx.save_for_backward(x, w)
        ctx.ftp = ftp
        ctx.has_bias = b is not None
        return matmul_nt(x, w, bias=b)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = ctx.ftp.gemm_allreduce(dy, w, b_mn=True) if ctx.needs_input_grad[0] else None
        dw = weight_grad(dy, x) if ctx.needs_input_grad[1] else None
        db = dy.float().sum(0).to(dy.dtype) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return dx, dw, db, None


def row_parallel(x: torch.Tensor, w: torch.Tensor, ftp: FusedTP) -> torch.Tensor:
    return _RowParallelFn.apply(x.reshape(-1, x.shape[-1]), w, ftp)


def column_parallel(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, ftp: FusedTP) -> torch.Tensor:
    return _ColumnParallelFn.apply(x.reshape(-1, x.shape[-1]), w, b, ftp)
