"""Weight-streaming tcgen05 decode GEMM (csrc/gemm_skinny.cu) against fp32
PyTorch: every token-tile width, split-K through the fp32 workspace (which must
be all zero again afterwards), bias, more rows than one launch takes."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B", [1, 17, 64, 130, 256, 300])
@pytest.mark.parametrize("N,K,bias", [(2560, 2048, True), (2048, 11008, False), (22016, 2048, False)])
def test_decode_linear_matches_fp32(B, N, K, bias):
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import decode_linear
    g = torch.Generator(device="cuda").manual_seed(B + N)
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    b = torch.randn(N, device="cuda", generator=g).bfloat16() if bias else None
    ws = torch.zeros(512 * N, device="cuda")
    for _ in range(2):   # the workspace is reused: the second call must not see the first's sums
        y = decode_linear(x, w, b, ws)
        torch.cuda.synchronize()
        check_errors()
        ref = x.float() @ w.float().t() + (b.float() if bias else 0)
        err = (y.float() - ref).abs().max().item()
        assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err
        assert torch.count_nonzero(ws) == 0


def test_decode_linear_without_split():
    from psrl_b200.ops.linear import decode_linear
    x = torch.randn(40, 2048, device="cuda").bfloat16()
    w = (torch.randn(151936, 2048, device="cuda") * 0.02).bfloat16()
    y = decode_linear(x, w)
    ref = x.float() @ w.float().t()
    assert (y.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
