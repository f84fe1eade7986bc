"""Paired-CTA tcgen05 GEMM (csrc/gemm_2sm.cu) against fp32 PyTorch references:
every operand layout (forward, data gradient, weight gradient), ragged M / N /
K edges, split-K accumulation, bias, the fused gate_up + SwiGLU epilogue, and
the autograd linear used by the model."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).bfloat16()


def _check(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    assert err <= tol * max(1.0, ref.abs().max().item()), f"max abs err {err}"


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 520, 200), (1000, 2560, 2048), (4096, 2048, 11008),
                                   (17, 8, 64), (513, 264, 72)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_matmul_nt_layouts(M, N, K, a_mn, b_mn):
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import matmul_nt
    A = _rand(M, K, seed=1, scale=0.5)
    B = _rand(N, K, seed=2, scale=0.5)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    if (a_mn and M % 8) or (b_mn and N % 8) or K % 8:
        pytest.skip("row stride not a multiple of 16 bytes")
    out = matmul_nt(a, b, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    check_errors()
    _check(out, A.float() @ B.float().t())


@pytest.mark.parametrize("splits", [1, 3, 8])
def test_matmul_nt_split_k_accumulates(splits):
    from psrl_b200.ops.linear import matmul_nt
    M, N, K = 640, 384, 4096
    A, B = _rand(K, M, seed=3, scale=0.3), _rand(K, N, seed=4, scale=0.3)   # MN-major, as in a weight gradient
    acc = torch.full((M, N), 1.5, device="cuda")
    matmul_nt(A, B, a_mn=True, b_mn=True, out=acc, splits=splits)
    ref = A.float().t() @ B.float() + 1.5
    torch.testing.assert_close(acc, ref, atol=2e-2, rtol=1e-2)


def test_bias_epilogue():
    from psrl_b200.ops.linear import matmul_nt
    x, w, b = _rand(700, 2048, seed=5), _rand(2560, 2048, seed=6, scale=0.02), _rand(2560, seed=7)
    out = matmul_nt(x, w, bias=b)
    _check(out, x.float() @ w.float().t() + b.float())


@pytest.mark.parametrize("M", [256, 999, 4096])
def test_gate_up_swiglu_fused(M):
    import torch.nn.functional as F
    from psrl_b200.ops import ext
    from psrl_b200.ops.gemm import _err
    I, H = 1408, 2048
    x, w = _rand(M, H, seed=8), _rand(2 * I, H, seed=9, scale=0.02)
    gu, h = ext().tc_gemm2_swiglu(x, w, 8, _err(x.device))
    ref = x.float() @ w.float().t()
    _check(gu, ref)
    g, u = ref.chunk(2, dim=-1)
    _check(h, F.silu(g) * u)


def test_linear_autograd_matches_fp32():
    from psrl_b200.ops.linear import gate_up_swiglu, linear
    M, H, I = 1500, 1024, 768
    x0 = _rand(M, H, seed=10)
    w1 = _rand(2 * I, H, seed=11, scale=0.03)
    w2 = _rand(H, I, seed=12, scale=0.03)
    b1 = _rand(H, seed=13)
    dy = _rand(M, H, seed=14)
    # tcgen05 path
    x = x0.clone().requires_grad_(True)
    p1, p2, pb = (w1.clone().requires_grad_(True), w2.clone().requires_grad_(True), b1.clone().requires_grad_(True))
    y = linear(gate_up_swiglu(x, p1), p2, pb)
    y.backward(dy)
    # fp32 reference
    xr = x0.float().requires_grad_(True)
    r1, r2, rb = (w1.float().requires_grad_(True), w2.float().requires_grad_(True), b1.float().requires_grad_(True))
    g, u = (xr @ r1.t()).chunk(2, dim=-1)
    yr = (torch.nn.functional.silu(g) * u) @ r2.t() + rb
    yr.backward(dy.float())
    _check(y, yr.detach(), 3e-2)
    for got, ref in ((x.grad, xr.grad), (p1.grad, r1.grad), (p2.grad, r2.grad), (pb.grad, rb.grad)):
        _check(got, ref, 3e-2)
