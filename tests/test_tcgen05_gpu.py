"""tcgen05/TMEM GEMM kernels against fp32 PyTorch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 520, 128), (1000, 2560, 2048), (37, 151936 // 8, 512)])
def test_tc_gemm_matches_matmul(M, N, K):
    from psrl_b200.ops.gemm import check_errors, tc_linear
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.5).bfloat16()
    y = tc_linear(x, w)
    torch.cuda.synchronize()
    check_errors()
    ref = x.float() @ w.float().t()
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 1e-2, float(rel)
    torch.testing.assert_close(y.float(), ref, atol=0.1 * K ** 0.5 / 8, rtol=2e-2)


@pytest.mark.parametrize("temp", [1.0, 0.7])
def test_tc_linear_logprob(temp):
    from psrl_b200.ops.gemm import check_errors, tc_linear_logprob
    g = torch.Generator(device="cuda").manual_seed(5)
    T, H, V = 333, 256, 5000 + 8
    h = (0.5 * torch.randn(T, H, device="cuda", generator=g)).bfloat16()
    W = (0.5 * torch.randn(V, H, device="cuda", generator=g)).bfloat16()
    lab = torch.randint(0, V, (T,), device="cuda", generator=g)
    lab[7] = -1
    lp, ent, lse = tc_linear_logprob(h, W, lab, temp)
    torch.cuda.synchronize()
    check_errors()
    logits = (h.float() @ W.float().t()) / temp
    logp = logits.log_softmax(-1)
    lpr = logp.gather(-1, lab.clamp_min(0)[:, None])[:, 0] * (lab >= 0)
    entr = -(logp.exp() * logp).sum(-1)
    torch.testing.assert_close(lse, logits.logsumexp(-1), atol=2e-2, rtol=1e-3)
    torch.testing.assert_close(lp, lpr, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(ent, entr, atol=5e-2, rtol=2e-2)
