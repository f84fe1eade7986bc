"""Small, fixed workloads for one-kernel profiler captures.

Each case allocates a few hundred MB at most (operands larger than L2 where
DRAM traffic matters), runs its kernel a few times and synchronises, so a
capture of one or two launches under a profiler ends within a minute.

    python -m psrl_b200.bench.profile_cases --case gemm_fwd
    python -m psrl_b200.bench.profile_cases --case attn

Cases:
  gemm_fwd   paired-CTA tcgen05 GEMM, x [16384, 2048] @ W[4096, 2048]^T
  gemm_wgrad same kernel as a weight gradient (both operands MN-major)
  gate_up    fused gate_up + SwiGLU epilogue, x [16384, 2048], W [22016, 2048]
  attn       tcgen05 varlen causal attention fwd + bwd, 6 x 1700 tokens, 16/2 heads
  decode     paged decode attention, B=256, context 1024, 16/2 heads
  skinny     weight-streaming decode GEMM, 128 rows: gate_up + SwiGLU (22016 x 2048)
             and QKV (2560 x 2048, K split over a 4-CTA cluster)
"""

from __future__ import annotations

import argparse

import torch


def _gemm(role: str, iters: int) -> None:
    from psrl_b200.ops.linear import matmul_nt, weight_grad
    M, N, K = 16384, 4096, 2048
    x = torch.randn(M, K, device="cuda").bfloat16()
    if role == "fwd":
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        for _ in range(iters):
            matmul_nt(x, w)
    else:
        dy = torch.randn(M, N, device="cuda").bfloat16()
        for _ in range(iters):
            weight_grad(dy, x)


def _gate_up(iters: int) -> None:
    from psrl_b200.ops.linear import gate_up_swiglu
    x = torch.randn(16384, 2048, device="cuda").bfloat16()
    w = (torch.randn(22016, 2048, device="cuda") * 0.02).bfloat16()
    for _ in range(iters):
        gate_up_swiglu(x, w)


def _attn(iters: int) -> None:
    from psrl_b200.ops import varlen_attention
    L, nseq, nq, nkv, d = 1700, 6, 16, 2, 128
    T = L * nseq
    qkv = torch.randn(T, (nq + 2 * nkv) * d, device="cuda").bfloat16().requires_grad_(True)
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device="cuda")
    for _ in range(iters):
        o = varlen_attention(qkv, cu, L, nq, nkv, d)
        o.backward(torch.ones_like(o))


def _decode(iters: int) -> None:
    from psrl_b200.ops import paged_decode_attention
    B, ctx, nq, nkv, bs, d = 256, 1024, 16, 2, 64, 128
    nblk = B * (ctx // bs)
    kc = torch.randn(nblk, nkv, bs, d, device="cuda").bfloat16()
    vc = torch.randn_like(kc)
    bt = torch.randperm(nblk, device="cuda").to(torch.int32).view(B, ctx // bs)
    lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(B, nq, d, device="cuda").bfloat16()
    for _ in range(iters):
        paged_decode_attention(q, kc, vc, bt, lens)


def _skinny(iters: int) -> None:
    from psrl_b200.ops.linear import decode_gate_up_swiglu, decode_linear
    x = torch.randn(128, 2048, device="cuda").bfloat16()
    w = (torch.randn(22016, 2048, device="cuda") * 0.02).bfloat16()
    wq = (torch.randn(2560, 2048, device="cuda") * 0.02).bfloat16()
    for _ in range(iters):
        decode_gate_up_swiglu(x, w)
        decode_linear(x, wq)


CASES = {"skinny": _skinny, "gemm_fwd": lambda n: _gemm("fwd", n), "gemm_wgrad": lambda n: _gemm("wgrad", n), "gate_up": _gate_up,
         "attn": _attn, "decode": _decode}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(CASES), required=True)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    CASES[args.case](args.iters)
    torch.cuda.synchronize()
    from psrl_b200.ops.gemm import check_errors
    check_errors()
    print(f"{args.case}: ok", flush=True)


if __name__ == "__main__":
    main()
