"""tcgen05 / TMEM causal varlen attention forward (csrc/attn_sm100.cu) against
the plain fp32 PyTorch attention of the same packed batch: ragged lengths
around the 128 / 256-row tile edges, GQA 8:1 and 7:1, and the log-sum-exp the
backward consumes."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(lens, nq, nkv, seed=0):
    d = 128
    T = sum(lens)
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = torch.randn(T, (nq + 2 * nkv) * d, device="cuda", generator=g).bfloat16()
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    return qkv, cu


def _ref(qkv, cu, nq, nkv, scale):
    d = 128
    T = qkv.shape[0]
    q = qkv[:, : nq * d].float().view(T, nq, d)
    k = qkv[:, nq * d:(nq + nkv) * d].float().view(T, nkv, d)
    v = qkv[:, (nq + nkv) * d:].float().view(T, nkv, d)
    outs, lses = [], []
    cl = cu.tolist()
    for i in range(len(cl) - 1):
        s, e = cl[i], cl[i + 1]
        if e == s:
            continue
        qs = q[s:e].transpose(0, 1)
        ks = k[s:e].transpose(0, 1).repeat_interleave(nq // nkv, 0)
        vs = v[s:e].transpose(0, 1).repeat_interleave(nq // nkv, 0)
        att = (qs @ ks.transpose(1, 2)) * scale
        mask = torch.ones(e - s, e - s, dtype=torch.bool, device="cuda").triu(1)
        att = att.masked_fill(mask, float("-inf"))
        lses.append(att.logsumexp(-1))
        outs.append((att.softmax(-1) @ vs).transpose(0, 1))
    return torch.cat(outs, 0).reshape(T, nq * d), torch.cat(lses, 1)


@pytest.mark.parametrize("lens,nq,nkv", [
    ([1, 17, 128, 129, 255, 256, 257, 300], 16, 2),
    ([1000, 513, 64], 16, 2),
    ([700, 129, 1], 28, 4),
    ([2048], 16, 2),
])
def test_fwd_matches_fp32(lens, nq, nkv):
    from psrl_b200.ops.attention import varlen_attention_fwd
    from psrl_b200.ops.gemm import check_errors
    qkv, cu = _case(lens, nq, nkv)
    scale = 1.0 / math.sqrt(128)
    o, lse = varlen_attention_fwd(qkv, cu, max(lens), nq, nkv, scale, want_lse=True)
    torch.cuda.synchronize()
    check_errors()
    ref_o, ref_lse = _ref(qkv, cu, nq, nkv, scale)
    torch.testing.assert_close(o.float(), ref_o, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, ref_lse, atol=1e-3, rtol=1e-3)


def test_fwd_large_logits_rescale():
    """Keys whose scores grow along the sequence force the lazily rescaled
    running maximum through several updates."""
    from psrl_b200.ops.attention import varlen_attention_fwd
    nq, nkv, L = 16, 2, 1024
    qkv, cu = _case([L], nq, nkv, seed=3)
    d = 128
    ramp = torch.linspace(0, 6, L, device="cuda")[:, None]
    qkv[:, nq * d:(nq + nkv) * d] = (qkv[:, nq * d:(nq + nkv) * d].float() * ramp).bfloat16()
    scale = 1.0 / math.sqrt(d)
    o, lse = varlen_attention_fwd(qkv, cu, L, nq, nkv, scale, want_lse=True)
    ref_o, ref_lse = _ref(qkv, cu, nq, nkv, scale)
    torch.testing.assert_close(o.float(), ref_o, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(lse, ref_lse, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("lens,nq,nkv", [
    ([1, 17, 128, 129, 255, 300], 16, 2),
    ([700, 129], 28, 4),
    ([1024], 16, 2),
])
def test_bwd_matches_fp32(lens, nq, nkv):
    from psrl_b200.ops import ext
    from psrl_b200.ops.attention import varlen_attention_fwd
    from psrl_b200.ops.gemm import _err, check_errors
    d = 128
    qkv, cu = _case(lens, nq, nkv, seed=5)
    T = qkv.shape[0]
    scale = 1.0 / math.sqrt(d)
    o, lse = varlen_attention_fwd(qkv, cu, max(lens), nq, nkv, scale, want_lse=True)
    g = torch.Generator(device="cuda").manual_seed(6)
    dout = torch.randn(T, nq * d, device="cuda", generator=g).bfloat16()
    dqkv = ext().attn_bwd_sm100(qkv, o, dout, lse, cu, max(lens), nq, nkv, scale, _err(qkv.device))
    torch.cuda.synchronize()
    check_errors()
    qf = qkv.float().requires_grad_(True)
    ref_o, _ = _ref(qf, cu, nq, nkv, scale)
    ref_o.backward(dout.float())
    ref = qf.grad
    for name, sl in (("dq", slice(0, nq * d)), ("dk", slice(nq * d, (nq + nkv) * d)), ("dv", slice((nq + nkv) * d, None))):
        got, want = dqkv[:, sl].float(), ref[:, sl]
        err = (got - want).abs().max().item()
        assert err <= 5e-2 * max(1.0, want.abs().max().item()), f"{name}: max abs err {err}"


@pytest.mark.parametrize("pairs,nq,nkv", [
    ([(128, 128), (100, 300), (257, 257)], 16, 2),
    ([(64, 1000), (200, 1700), (130, 131), (1, 77)], 16, 2),
    ([(300, 812)], 28, 4),
])
def test_attention_kv_matches_fp32(pairs, nq, nkv):
    """Queries that are the last Lq of Lk key positions (context-parallel
    chunks): forward, log-sum-exp and the q / kv gradients against fp32."""
    from psrl_b200.ops.attention import attention_kv, attention_kv_ref
    from psrl_b200.ops.gemm import check_errors
    d = 128
    Tq, Tk = sum(p[0] for p in pairs), sum(p[1] for p in pairs)
    g = torch.Generator(device="cuda").manual_seed(len(pairs))
    q = torch.randn(Tq, nq * d, device="cuda", generator=g).bfloat16().requires_grad_(True)
    kv = torch.randn(Tk, 2 * nkv * d, device="cuda", generator=g).bfloat16().requires_grad_(True)
    cu_q = torch.tensor([0] + list(torch.tensor([p[0] for p in pairs]).cumsum(0)), dtype=torch.int32, device="cuda")
    cu_k = torch.tensor([0] + list(torch.tensor([p[1] for p in pairs]).cumsum(0)), dtype=torch.int32, device="cuda")
    scale = 1.0 / math.sqrt(d)
    o = attention_kv(q, kv, cu_q, cu_k, max(p[0] for p in pairs), max(p[1] for p in pairs), nq, nkv, d, scale)
    dout = torch.randn(Tq, nq * d, device="cuda", generator=g).bfloat16()
    o.backward(dout)
    torch.cuda.synchronize()
    check_errors()
    qf = q.detach().float().requires_grad_(True)
    kvf = kv.detach().float().requires_grad_(True)
    ref = attention_kv_ref(qf.view(Tq, nq, d), kvf[:, : nkv * d].reshape(Tk, nkv, d),
                           kvf[:, nkv * d:].reshape(Tk, nkv, d), cu_q, cu_k, scale).reshape(Tq, nq * d)
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)
    ref.backward(dout.float())
    for name, got, want in (("dq", q.grad, qf.grad), ("dkv", kv.grad, kvf.grad)):
        err = (got.float() - want).abs().max().item()
        assert err <= 5e-2 * max(1.0, want.abs().max().item()), f"{name}: max abs err {err}"
