"""Fused MoE kernels (router top-k, permutation, gather/combine, tcgen05
grouped expert GEMM) against fp32 PyTorch references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_route_matches_softmax_topk():
    from psrl_b200.ops import moe
    g = torch.Generator(device="cuda").manual_seed(0)
    T, E, k = 517, 128, 8
    logits = torch.randn(T, E, device="cuda", generator=g)
    prior = torch.randn(E, device="cuda", generator=g) * 0.5
    w, ids, counts = moe.route(logits, prior, k, renorm=True)
    wr, idr = moe.route_ref(logits, prior, k, renorm=True)
    assert torch.equal(ids, idr)
    torch.testing.assert_close(w, wr, atol=1e-5, rtol=1e-4)
    assert torch.equal(counts.long(), torch.bincount(idr.reshape(-1).long(), minlength=E))


@pytest.mark.parametrize("counts", [[0, 5, 300, 0, 128, 1, 257, 64], [1000, 0, 0, 3]])
def test_grouped_gemm_matches_per_expert_matmul(counts):
    from psrl_b200.ops._ext import ext
    from psrl_b200.ops.gemm import check_errors
    g = torch.Generator(device="cuda").manual_seed(len(counts))
    E, N, K = len(counts), 1536, 2048
    R = sum(counts)
    x = (torch.randn(R, K, device="cuda", generator=g) * 0.5).bfloat16()
    w = (torch.randn(E, N, K, device="cuda", generator=g) * 0.05).bfloat16()
    seg = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ext().tc_grouped_gemm(x, w, seg, err)
    torch.cuda.synchronize()
    check_errors()
    assert int(err.item()) == 0
    ref = torch.empty(R, N, device="cuda")
    s = 0
    for e, c in enumerate(counts):
        ref[s:s + c] = x[s:s + c].float() @ w[e].float().t()
        s += c
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 1e-2, float(rel)


def _moe_case(T=200, E=16, h=256, I=128, k=4, seed=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(T, h, device="cuda", generator=g) * 0.5).bfloat16()
    logits = torch.randn(T, E, device="cuda", generator=g)
    prior = torch.randn(E, device="cuda", generator=g) * 0.3
    w13 = (torch.randn(E, 2 * I, h, device="cuda", generator=g) * 0.05).bfloat16()
    w2 = (torch.randn(E, h, I, device="cuda", generator=g) * 0.05).bfloat16()
    return x, logits, prior, w13, w2, k


def test_moe_mlp_matches_local_path():
    from psrl_b200.ops import moe
    from psrl_b200.parallel.moe import moe_forward_local
    x, logits, prior, w13, w2, k = _moe_case()
    y = moe.moe_mlp(x, logits, prior, w13, w2, k, renorm=True)
    w, ids = moe.route_ref(logits, prior, k, True)
    ref = moe_forward_local(x.float(), w.float(), ids.long(), w13.float(), w2.float())
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 2e-2, float(rel)


def test_moe_mlp_gradients():
    from psrl_b200.ops import moe
    from psrl_b200.parallel.moe import moe_forward_local
    x, logits, prior, w13, w2, k = _moe_case(T=96, seed=4)
    outs = []
    for fused in (True, False):
        xx = x.float().clone().requires_grad_(True) if not fused else x.clone().requires_grad_(True)
        lg = logits.clone().requires_grad_(True)
        a = w13.clone().requires_grad_(True) if fused else w13.float().clone().requires_grad_(True)
        b = w2.clone().requires_grad_(True) if fused else w2.float().clone().requires_grad_(True)
        if fused:
            y = moe.moe_mlp(xx, lg, prior, a, b, k, renorm=True)
        else:
            z = (lg + prior).softmax(-1)
            wk, ids = z.topk(k, -1)
            wk = wk / wk.sum(-1, keepdim=True)
            y = moe_forward_local(xx, wk, ids, a, b)
        (y.float() * torch.linspace(-1, 1, y.shape[1], device="cuda")).sum().backward()
        outs.append([t.grad.float() for t in (xx, lg, a, b)])
    for gf, gr in zip(*outs):
        rel = (gf - gr).norm() / gr.norm().clamp_min(1e-12)
        assert rel < 5e-2, float(rel)


def test_moe_model_fused_path_matches_local_path(monkeypatch):
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.ops import moe
    a = PRESETS["tiny-moe"]
    m = build_model(a, "cuda", torch.bfloat16, seed=2)
    g = torch.Generator(device="cuda").manual_seed(0)
    lens = [37, 64, 5]
    ids = torch.randint(0, a.vocab_size, (sum(lens),), device="cuda", generator=g)
    pos, cu, mx = packed_positions(lens, "cuda")
    with torch.no_grad():
        h_fused = m.hidden_states(ids, pos, cu, mx).float()
        monkeypatch.setattr(moe, "supported", lambda *args: False)
        h_local = m.hidden_states(ids, pos, cu, mx).float()
    rel = (h_fused - h_local).norm() / h_local.norm()
    assert rel < 3e-2, float(rel)


def test_moe_rollout_engine_decodes_with_graphs():
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    a = PRESETS["tiny-moe"]
    m = build_model(a, "cuda", torch.bfloat16, seed=2)
    eng = RolloutEngine(a, EngineWeights.from_model(m), max_num_seqs=8, max_model_len=256, block_size=64,
                        kv_cache_gb=0.5, use_cuda_graph=True)
    for i in range(5):
        eng.add_request(GenRequest(i, list(range(3, 3 + 10 + i)), SamplingParams(max_tokens=12, ignore_eos=True,
                                                                                seed=i)))
    outs = []
    while eng.has_unfinished():
        outs += eng.step()
    assert len(outs) == 5 and all(len(o.output_ids) == 12 for o in outs)
    assert all(0 <= t < a.vocab_size for o in outs for t in o.output_ids)
