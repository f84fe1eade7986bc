"""Stream-K weight-streaming tcgen05 decode GEMM (csrc/gemm_skinny.cu) against
fp32 PyTorch: every token-tile width, tiles shared by several CTAs (the fp32
workspace and the tickets must be all zero again afterwards), bias, the fused
SwiGLU epilogue, CTA counts that split tiles unevenly, more rows than one launch
takes."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_tol(ref):
    return 2e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("B", [1, 17, 64, 130, 256, 300])
@pytest.mark.parametrize("N,K,bias", [(2560, 2048, True), (2048, 11008, False), (22016, 2048, False), (1000, 512, True)])
def test_decode_linear_matches_fp32(B, N, K, bias):
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import DecodeWorkspace, decode_linear
    g = torch.Generator(device="cuda").manual_seed(B + N)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16() if bias else None
    ws = DecodeWorkspace(N, "cuda")
    ref = x.float() @ w.float().t() + (b.float() if bias else 0)
    for _ in range(2):   # the workspace is reused: the second call must not see the first's sums
        y = decode_linear(x, w, b, ws)
        torch.cuda.synchronize()
        check_errors()
        err = (y.float() - ref).abs().max().item()
        assert err <= _ref_tol(ref), err
        assert torch.count_nonzero(ws.acc) == 0 and torch.count_nonzero(ws.tickets) == 0


@pytest.mark.parametrize("grid", [1, 7, 37, 148, 1000])
def test_decode_linear_grid_sizes(grid):
    """Unit ranges that start and end mid-tile, a tile spread over many CTAs,
    one CTA doing everything, more CTAs than units."""
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import DecodeWorkspace, decode_linear
    g = torch.Generator(device="cuda").manual_seed(grid)
    x = torch.randn(48, 1024, device="cuda", generator=g).bfloat16()
    w = (torch.randn(640, 1024, device="cuda", generator=g) * 0.02).bfloat16()
    b = torch.randn(640, device="cuda", generator=g).bfloat16()
    ws = DecodeWorkspace(640, "cuda")
    y = decode_linear(x, w, b, ws, grid=grid)
    torch.cuda.synchronize()
    check_errors()
    ref = x.float() @ w.float().t() + b.float()
    assert (y.float() - ref).abs().max().item() <= _ref_tol(ref)
    assert torch.count_nonzero(ws.acc) == 0 and torch.count_nonzero(ws.tickets) == 0


@pytest.mark.parametrize("B", [3, 64, 200, 256])
@pytest.mark.parametrize("grid", [0, 50])
def test_decode_gate_up_swiglu_matches_fp32(B, grid):
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import DecodeWorkspace, decode_gate_up_swiglu
    I, K = 11008, 2048
    g = torch.Generator(device="cuda").manual_seed(B)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.02).bfloat16()
    ws = DecodeWorkspace(2 * I, "cuda")
    gu = x.float() @ w.float().t()
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    for _ in range(2):
        h = decode_gate_up_swiglu(x, w, ws, grid=grid)
        torch.cuda.synchronize()
        check_errors()
        assert h.shape == (B, I)
        assert (h.float() - ref).abs().max().item() <= _ref_tol(ref)
        assert torch.count_nonzero(ws.acc) == 0 and torch.count_nonzero(ws.tickets) == 0


def test_decode_linear_vocab_head():
    from psrl_b200.ops.linear import decode_linear
    x = torch.randn(40, 2048, device="cuda").bfloat16()
    w = (torch.randn(151936, 2048, device="cuda") * 0.02).bfloat16()
    y = decode_linear(x, w)
    ref = x.float() @ w.float().t()
    assert (y.float() - ref).abs().max().item() <= _ref_tol(ref)
