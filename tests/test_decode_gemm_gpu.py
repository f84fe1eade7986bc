"""Weight-streaming tcgen05 decode GEMM (csrc/gemm_skinny.cu) against fp32
PyTorch: every token-tile width, the K loop split over clusters of 1, 2, 4
and 8 CTAs (partials reduced through distributed shared memory), bias, the
fused SwiGLU epilogue, ragged feature counts, more rows than one launch takes."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _tol(ref):
    return 2e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("B", [1, 17, 64, 130, 256, 300])
@pytest.mark.parametrize("N,K,bias", [(2560, 2048, True), (2048, 11008, False), (22016, 2048, False), (1000, 512, True)])
def test_decode_linear_matches_fp32(B, N, K, bias):
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import decode_linear
    g = torch.Generator(device="cuda").manual_seed(B + N)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16() if bias else None
    ref = x.float() @ w.float().t() + (b.float() if bias else 0)
    y = decode_linear(x, w, b)
    torch.cuda.synchronize()
    check_errors()
    assert (y.float() - ref).abs().max().item() <= _tol(ref)


@pytest.mark.parametrize("split", [1, 2, 4, 8])
@pytest.mark.parametrize("B", [5, 128, 256])
def test_decode_linear_cluster_splits(split, B):
    """Every cluster size, token counts that leave some CTAs of the cluster
    without a share of the reduction."""
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import decode_linear
    g = torch.Generator(device="cuda").manual_seed(split * 1000 + B)
    x = torch.randn(B, 1024, device="cuda", generator=g).bfloat16()
    w = (torch.randn(640, 1024, device="cuda", generator=g) * 0.02).bfloat16()
    b = torch.randn(640, device="cuda", generator=g).bfloat16()
    y = decode_linear(x, w, b, split=split)
    torch.cuda.synchronize()
    check_errors()
    ref = x.float() @ w.float().t() + b.float()
    assert (y.float() - ref).abs().max().item() <= _tol(ref)


@pytest.mark.parametrize("B", [3, 64, 200, 256])
@pytest.mark.parametrize("split", [0, 2])
def test_decode_gate_up_swiglu_matches_fp32(B, split):
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import decode_gate_up_swiglu
    I, K = 11008, 2048
    g = torch.Generator(device="cuda").manual_seed(B)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.02).bfloat16()
    gu = x.float() @ w.float().t()
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    h = decode_gate_up_swiglu(x, w, split=split)
    torch.cuda.synchronize()
    check_errors()
    assert h.shape == (B, I)
    assert (h.float() - ref).abs().max().item() <= _tol(ref)


def test_decode_linear_vocab_head():
    from psrl_b200.ops.linear import decode_linear
    x = torch.randn(40, 2048, device="cuda").bfloat16()
    w = (torch.randn(151936, 2048, device="cuda") * 0.02).bfloat16()
    y = decode_linear(x, w)
    ref = x.float() @ w.float().t()
    assert (y.float() - ref).abs().max().item() <= _tol(ref)
