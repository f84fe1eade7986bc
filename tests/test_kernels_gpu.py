"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ext():
    from psrl_b200.ops import ext
    return ext()


def test_extension_loaded():
    e = _ext()
    assert hasattr(e, "attn_decode")


# ------------------------------------------------------------------ rmsnorm
@pytest.mark.parametrize("h", [512, 2048, 3584])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm_fwd_bwd(h, with_res):
    from psrl_b200.ops import rms_norm, rms_norm_ref
    torch.manual_seed(0)
    x = torch.randn(37, h, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    r = torch.randn(37, h, device=DEV, dtype=torch.bfloat16, requires_grad=True) if with_res else None
    w = (1 + 0.1 * torch.randn(h, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    y, s = rms_norm(x, w, 1e-6, r)
    xf = x.detach().float().requires_grad_(True)
    rf = r.detach().float().requires_grad_(True) if with_res else None
    wf = w.detach().float().requires_grad_(True)
    sf = xf + rf if with_res else xf
    yr = sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=3e-2)
    gy = torch.randn_like(yr)
    gs = torch.randn_like(yr) if with_res else None
    loss = (y.float() * gy).sum() + ((s.float() * gs).sum() if with_res else 0)
    loss.backward()
    lr = (yr * gy).sum() + ((sf * gs).sum() if with_res else 0)
    lr.backward()
    torch.testing.assert_close(x.grad.float(), xf.grad, atol=5e-2, rtol=5e-2)
    torch.testing.assert_close(w.grad.float(), wf.grad, atol=0.5, rtol=5e-2)
    if with_res:
        torch.testing.assert_close(r.grad.float(), rf.grad, atol=5e-2, rtol=5e-2)


# --------------------------------------------------------------------- rope
@pytest.mark.parametrize("d", [64, 128])
def test_rope_and_cache_write(d):
    from psrl_b200.ops.rope import apply_rope_ref, rope_qkv_, rope_tables
    torch.manual_seed(0)
    nq, nkv, T = 4, 2, 50
    qkv = torch.randn(T, (nq + 2 * nkv) * d, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 5000, (T,), device=DEV, dtype=torch.int32)
    ref = qkv.clone().float()
    cos, sin = rope_tables(1e6, d, 65536, DEV)
    q = apply_rope_ref(ref[:, : nq * d].view(T, nq, d), pos, cos, sin)
    k = apply_rope_ref(ref[:, nq * d:(nq + nkv) * d].view(T, nkv, d), pos, cos, sin)
    bs = 16
    kc = torch.zeros(8, nkv, bs, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(8 * bs, device=DEV)[:T].int()
    slots[3] = -1
    out = qkv.clone()
    rope_qkv_(out, pos, nq, nkv, d, 1e6, k_cache=kc, v_cache=vc, slots=slots)
    torch.testing.assert_close(out[:, : nq * d].float().view(T, nq, d), q, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(out[:, nq * d:(nq + nkv) * d].float().view(T, nkv, d), k, atol=2e-2, rtol=2e-2)
    v = qkv[:, (nq + nkv) * d:].view(T, nkv, d)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        torch.testing.assert_close(kc[s // bs, :, s % bs].float(), out[t, nq * d:(nq + nkv) * d].float().view(nkv, d))
        torch.testing.assert_close(vc[s // bs, :, s % bs], v[t])
    # inverse rotation restores the input
    back = out.clone()
    rope_qkv_(back, pos, nq, nkv, d, 1e6, inverse=True)
    torch.testing.assert_close(back.float(), qkv.float(), atol=3e-2, rtol=3e-2)


# ------------------------------------------------------------------- swiglu
def test_swiglu_fwd_bwd():
    from psrl_b200.ops import swiglu
    torch.manual_seed(0)
    gu = torch.randn(33, 2 * 1024, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    y = swiglu(gu)
    gf = gu.detach().float().requires_grad_(True)
    g, u = gf.chunk(2, -1)
    yr = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(y.float(), yr, atol=2e-2, rtol=2e-2)
    go = torch.randn_like(yr)
    (y.float() * go).sum().backward()
    (yr * go).sum().backward()
    torch.testing.assert_close(gu.grad.float(), gf.grad, atol=5e-2, rtol=5e-2)


# -------------------------------------------------------------------- adamw
@pytest.mark.parametrize("gdtype", [torch.float32, torch.bfloat16])
def test_adamw(gdtype):
    from psrl_b200.ops import adamw_, adamw_ref
    torch.manual_seed(0)
    n = 4096 + 64
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV).to(gdtype)
    m = torch.randn(n, device=DEV).abs() * 0.1
    v = torch.randn(n, device=DEV).abs() * 0.1
    p2, m2, v2 = p.clone(), m.clone(), v.clone()
    p16 = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    coef = torch.tensor([0.5], device=DEV)
    adamw_(p, g, m, v, p16, 1e-3, 0.9, 0.999, 1e-8, 0.1, 3, coef, 0.25)
    adamw_ref(p2, g.float(), m2, v2, None, 1e-3, 0.9, 0.999, 1e-8, 0.1, 3, 0.125)
    torch.testing.assert_close(p, p2, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(m, m2, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(v, v2, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(p16.float(), p2, atol=1e-2, rtol=1e-2)


def test_grad_norm_and_clip():
    from psrl_b200.ops import NormAccumulator
    torch.manual_seed(0)
    xs = [torch.randn(1000 + i * 37, device=DEV) for i in range(5)] + [torch.randn(333, device=DEV).bfloat16()]
    acc = NormAccumulator(DEV)
    for x in xs:
        acc.add(x)
    ref = math.sqrt(sum(float(x.float().pow(2).sum()) for x in xs))
    coef, nrm = acc.clip_coef(1.0)
    assert abs(float(nrm) - ref) / ref < 1e-4
    assert abs(float(coef) - min(1.0, 1.0 / (ref + 1e-6))) < 1e-5


# ------------------------------------------------------------------ logprob
@pytest.mark.parametrize("temp", [1.0, 0.7])
def test_linear_logprob_fwd_bwd(temp):
    from psrl_b200.ops import linear_logprob
    torch.manual_seed(0)
    T, H, V = 300, 256, 5000 + 8
    h = (0.5 * torch.randn(T, H, device=DEV)).bfloat16().requires_grad_(True)
    W = (0.5 * torch.randn(V, H, device=DEV)).bfloat16().requires_grad_(True)
    lab = torch.randint(0, V, (T,), device=DEV)
    lab[5] = -1
    lp, ent = linear_logprob(h, W, lab, temp, chunk=128)
    hf = h.detach().float().requires_grad_(True)
    Wf = W.detach().float().requires_grad_(True)
    logits = (hf.bfloat16().float() @ Wf.t()) / temp
    logp = logits.log_softmax(-1)
    lpr = logp.gather(-1, lab.clamp_min(0)[:, None])[:, 0] * (lab >= 0)
    entr = -(logp.exp() * logp).sum(-1)
    torch.testing.assert_close(lp, lpr, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(ent, entr, atol=5e-2, rtol=2e-2)
    g1, g2 = torch.randn(T, device=DEV), torch.randn(T, device=DEV)
    ((lp * g1).sum() + (ent * g2).sum()).backward()
    ((lpr * g1).sum() + (entr * g2).sum()).backward()
    # d logits are materialised in bf16 for the two backward GEMMs: compare with a
    # bf16-appropriate criterion (relative Frobenius error) plus a loose elementwise bound
    for got, ref in ((h.grad.float(), hf.grad), (W.grad.float(), Wf.grad)):
        rel = (got - ref).norm() / ref.norm()
        assert rel < 2e-2, float(rel)
        torch.testing.assert_close(got, ref, atol=0.3, rtol=0.1)


def test_linear_logprob_full_vocab_gradients():
    """Training LM head at the Qwen vocabulary (V = 151936): forward through the
    fused log-sum-exp kernel, backward through chunked tcgen05 GEMMs, against
    fp32 autograd."""
    from psrl_b200.ops import linear_logprob
    torch.manual_seed(1)
    T, H, V = 1024, 2048, 151936
    h = (0.5 * torch.randn(T, H, device=DEV)).bfloat16().requires_grad_(True)
    W = (0.02 * torch.randn(V, H, device=DEV)).bfloat16().requires_grad_(True)
    lab = torch.randint(0, V, (T,), device=DEV)
    lp, ent = linear_logprob(h, W, lab, 1.0, chunk=512)
    hf = h.detach().float().requires_grad_(True)
    Wf = W.detach().float().requires_grad_(True)
    logp = (hf @ Wf.t()).log_softmax(-1)
    lpr = logp.gather(-1, lab[:, None])[:, 0]
    entr = -(logp.exp() * logp).sum(-1)
    torch.testing.assert_close(lp, lpr, atol=3e-2, rtol=1e-2)
    torch.testing.assert_close(ent, entr, atol=3e-2, rtol=1e-2)
    g = torch.randn(T, device=DEV)
    (lp * g).sum().backward()
    (lpr * g).sum().backward()
    for got, ref in ((h.grad.float(), hf.grad), (W.grad.float(), Wf.grad)):
        rel = (got - ref).norm() / ref.norm()
        assert rel < 2e-2, float(rel)


# ----------------------------------------------------------------- sampling
def test_sampler_greedy_and_logprob():
    from psrl_b200.ops import sample
    torch.manual_seed(0)
    B, V = 64, 151936
    logits = torch.randn(B, V, device=DEV).bfloat16()
    temps = torch.zeros(B, device=DEV)
    tok, lp = sample(logits, temps, torch.arange(B, device=DEV), torch.zeros(B, device=DEV, dtype=torch.int32))
    assert torch.equal(tok, logits.float().argmax(-1))
    ref = logits.float().log_softmax(-1).gather(-1, tok[:, None])[:, 0]
    torch.testing.assert_close(lp, ref, atol=2e-3, rtol=1e-3)


def test_sampler_distribution():
    from psrl_b200.ops import sample
    V = 8
    probs = torch.tensor([0.4, 0.2, 0.1, 0.1, 0.08, 0.06, 0.04, 0.02])
    N = 40000
    logits = probs.log()[None].repeat(N, 1).to(DEV)
    temps = torch.ones(N, device=DEV)
    seeds = torch.full((N,), 7, device=DEV, dtype=torch.long)
    streams = torch.arange(N, device=DEV, dtype=torch.int32)
    tok, lp = sample(logits, temps, seeds, streams)
    freq = torch.bincount(tok.cpu(), minlength=V).float() / N
    assert (freq - probs).abs().max() < 0.015
    torch.testing.assert_close(lp.cpu(), probs.log()[tok.cpu()], atol=1e-4, rtol=1e-4)


# ---------------------------------------------------------------- attention
def _qkv(T, nq, nkv, d=128, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(T, (nq + 2 * nkv) * d, device=DEV, generator=g).bfloat16()


@pytest.mark.parametrize("lens,nq,nkv", [([1, 17, 64, 65, 200], 4, 2), ([300, 7, 128], 16, 2), ([130, 70], 28, 4)])
def test_varlen_attention_fwd_bwd(lens, nq, nkv):
    from psrl_b200.ops import varlen_attention, varlen_attention_ref
    d = 128
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    qkv = _qkv(T, nq, nkv).requires_grad_(True)
    o = varlen_attention(qkv, cu, max(lens), nq, nkv, d)
    qf = qkv.detach().float().requires_grad_(True)
    q = qf[:, : nq * d].view(T, nq, d)
    k = qf[:, nq * d:(nq + nkv) * d].view(T, nkv, d)
    v = qf[:, (nq + nkv) * d:].view(T, nkv, d)
    from psrl_b200.ops.attention import _ref_autograd
    orf = _ref_autograd(q, k, v, cu, 1 / math.sqrt(d)).reshape(T, -1)
    torch.testing.assert_close(o.float(), orf, atol=2e-2, rtol=2e-2)
    ref2 = varlen_attention_ref(q.detach(), k.detach(), v.detach(), cu, 1 / math.sqrt(d)).reshape(T, -1)
    torch.testing.assert_close(o.float(), ref2.float(), atol=2e-2, rtol=2e-2)
    go = torch.randn_like(orf)
    (o.float() * go).sum().backward()
    (orf * go).sum().backward()
    torch.testing.assert_close(qkv.grad.float(), qf.grad, atol=5e-2, rtol=5e-2)


def _paged_setup(ctx_lens, nkv, d=128, bs=16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    nblocks = sum((c + bs - 1) // bs for c in ctx_lens) + 4
    kc = torch.randn(nblocks, nkv, bs, d, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblocks, nkv, bs, d, device=DEV, generator=g).bfloat16()
    perm = torch.randperm(nblocks, generator=torch.Generator().manual_seed(seed)).tolist()
    maxb = max((c + bs - 1) // bs for c in ctx_lens)
    bt = torch.zeros(len(ctx_lens), maxb + 2, dtype=torch.int32)
    k = 0
    for i, c in enumerate(ctx_lens):
        nb = (c + bs - 1) // bs
        bt[i, :nb] = torch.tensor(perm[k: k + nb])
        k += nb
    return kc, vc, bt.to(DEV)


@pytest.mark.parametrize("bs", [16, 64])
def test_paged_prefill(bs):
    from psrl_b200.ops import paged_prefill_attention
    from psrl_b200.ops.attention import paged_attention_ref
    nq, nkv, d = 16, 2, 128
    ctx = [70, 200, 64, 1]
    qlen = [70, 33, 1, 1]
    kc, vc, bt = _paged_setup(ctx, nkv, d, bs)
    T = sum(qlen)
    q = torch.randn(T, nq, d, device=DEV).bfloat16()
    cu = torch.tensor([0] + list(torch.tensor(qlen).cumsum(0)), dtype=torch.int32, device=DEV)
    lens = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    o = paged_prefill_attention(q, kc, vc, cu, lens, bt, max(qlen))
    r = paged_attention_ref(q, kc, vc, cu, lens, bt, 1 / math.sqrt(d))
    torch.testing.assert_close(o.float(), r.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("splits", [1, 3, 8])
@pytest.mark.parametrize("nq,nkv", [(16, 2), (28, 4)])
def test_paged_decode(splits, nq, nkv):
    from psrl_b200.ops import paged_decode_attention
    from psrl_b200.ops.attention import paged_attention_ref
    d, bs = 128, 64
    ctx = [1, 63, 64, 65, 700, 1500]
    kc, vc, bt = _paged_setup(ctx, nkv, d, bs, seed=3)
    B = len(ctx)
    q = torch.randn(B, nq, d, device=DEV).bfloat16()
    lens = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    o = paged_decode_attention(q, kc, vc, bt, lens, splits=splits)
    cu = torch.arange(B + 1, dtype=torch.int32, device=DEV)
    r = paged_attention_ref(q, kc, vc, cu, lens, bt, 1 / math.sqrt(d))
    torch.testing.assert_close(o.float(), r.float(), atol=2e-2, rtol=2e-2)


# -------------------------------------------------------------- end to end
@pytest.mark.parametrize("chunk,decode_gemm", [(96, "library"), (1024, "library"), (1024, "tcgen05")])
def test_engine_greedy_matches_recompute_gpu(chunk, decode_gemm):
    # chunk 96: every prefill chunk on the library GEMM path; 1024: prefill
    # chunks of >= 256 rows run on the paired tcgen05 GEMM and fused SwiGLU
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    a = PRESETS["tiny128"]
    m = build_model(a, DEV, torch.bfloat16, seed=1)
    w = EngineWeights.from_model(m)
    eng = RolloutEngine(a, w, max_num_seqs=8, max_model_len=1024, block_size=64, max_num_batched_tokens=chunk,
                        num_blocks=96, use_cuda_graph=True, decode_gemm=decode_gemm)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, a.vocab_size, (n,), generator=g).tolist() for n in (5, 70, 330, 9)]
    for i, p in enumerate(prompts):
        eng.add_request(GenRequest(i, p, SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True)))
    outs = {}
    while eng.has_unfinished():
        for o in eng.step():
            outs[o.request_id] = o
    agree = 0
    total = 0
    for i, p in enumerate(prompts):
        toks = list(p) + outs[i].output_ids
        pos, cu, mx = packed_positions([len(toks) - 1], DEV)
        with torch.no_grad():
            lg = m.logits(torch.tensor(toks[:-1], device=DEV), pos, cu, mx)
        pred = lg.argmax(-1)[len(p) - 1:].tolist()
        agree += sum(int(x == y) for x, y in zip(pred, outs[i].output_ids))
        total += len(pred)
    # bf16 paths differ slightly (paged vs packed kernels); near-ties may flip
    assert agree / total > 0.9, (agree, total)


def test_rl_step_gpu_tiny():
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "model.preset=tiny128", "model.dtype=bf16", "trainer.device=cuda", "rollout.cuda_graph=true",
        "data.kind=synthetic_tokens", "data.prompt_len_min=16", "data.prompt_len_max=64",
        "data.response_len_mu=3.0", "data.response_len_sigma=0.5", "data.response_len_cap=64",
        "reward.kind=bernoulli_hash", "rollout.ignore_eos=true", "model.enable_gradient_checkpointing=true"])
    t = RLTrainer(cfg)
    for _ in range(3):
        m = t.step()
        assert m["num_trajectories"] == 32
        assert math.isfinite(m["actor/pg_loss"]) and math.isfinite(m["actor/grad_norm"])
    t.stop_rollout()
    assert t.ps.get_ps_model_version() == 3
    assert t.engine.version in (2, 3)


@pytest.mark.parametrize("nq,nkv", [(16, 2), (28, 4)])
def test_paged_decode_long_context(nq, nkv):
    """Decode over 8k-token contexts (the response cap of the DAPO recipe),
    default split choice, scattered pages, against the fp32 reference."""
    from psrl_b200.ops import paged_decode_attention
    from psrl_b200.ops.attention import paged_attention_ref
    d, bs = 128, 64
    ctx = [8192, 8000, 4097, 6000]
    kc, vc, bt = _paged_setup(ctx, nkv, d, bs, seed=5)
    B = len(ctx)
    q = torch.randn(B, nq, d, device=DEV).bfloat16()
    lens = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    o = paged_decode_attention(q, kc, vc, bt, lens)
    cu = torch.arange(B + 1, dtype=torch.int32, device=DEV)
    r = paged_attention_ref(q, kc, vc, cu, lens, bt, 1 / math.sqrt(d))
    torch.testing.assert_close(o.float(), r.float(), atol=2e-2, rtol=2e-2)


def test_engine_long_prompt_matches_recompute_gpu():
    """An 8k-token prompt through chunked prefill (tcgen05 projections) and
    CUDA-graph decode: greedy tokens agree with a packed recompute."""
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    a = PRESETS["tiny128"]
    m = build_model(a, DEV, torch.bfloat16, seed=4)
    eng = RolloutEngine(a, EngineWeights.from_model(m), max_num_seqs=4, max_model_len=8400, block_size=64,
                        max_num_batched_tokens=2048, kv_cache_gb=1.0, use_cuda_graph=True)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(3, a.vocab_size, (n,), generator=g).tolist() for n in (8192, 3000)]
    for i, p in enumerate(prompts):
        eng.add_request(GenRequest(i, p, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)))
    outs = {}
    while eng.has_unfinished():
        for o in eng.step():
            outs[o.request_id] = o
    agree = total = 0
    for i, p in enumerate(prompts):
        toks = list(p) + outs[i].output_ids
        pos, cu, mx = packed_positions([len(toks) - 1], DEV)
        with torch.no_grad():
            lg = m.logits(torch.tensor(toks[:-1], device=DEV), pos, cu, mx)
        pred = lg.argmax(-1)[len(p) - 1:].tolist()
        agree += sum(int(x == y) for x, y in zip(pred, outs[i].output_ids))
        total += len(pred)
    assert agree / total > 0.85, (agree, total)


def test_policy_step_gpu_matches_cpu_fp32():
    """One DAPO update of the same trajectories on the GPU (bf16, tcgen05
    kernels) and on the CPU (fp32 PyTorch): same loss and gradient norm within
    bf16 tolerance, parameters moved the same way."""
    import copy
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS
    from psrl_b200.trainer.actor import PolicyWorker
    from psrl_b200.trainer.batch import Trajectory
    a = PRESETS["tiny128"]
    g = torch.Generator().manual_seed(8)
    trajs = []
    for i, (P, R) in enumerate(((40, 300), (17, 129), (300, 64), (5, 500))):
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=torch.randint(0, a.vocab_size, (P,), generator=g).tolist(),
                                response_ids=torch.randint(0, a.vocab_size, (R,), generator=g).tolist(),
                                rollout_logprobs=(-torch.rand(R, generator=g) - 7.0).tolist()))
        trajs[-1].advantage = float(torch.randn(1, generator=g))
    res = {}
    init = None
    for dev, dt in (("cpu", "fp32"), ("cuda", "bf16")):
        cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"model.dtype={dt}", "actor.optim.lr=1e-3",
                                                             "actor.ppo_mini_batch_size=4"])
        w = PolicyWorker(cfg, a, dev, seed=3)
        # random init draws from the device's generator: give both workers the CPU weights
        if init is None:
            init = {n: p.detach().clone() for n, p in w.model.named_parameters()}
        else:
            with torch.no_grad():
                for n, p in w.model.named_parameters():
                    p.copy_(init[n])
            w.dp.sync_master_from_params()
        ts = copy.deepcopy(trajs)
        w.compute_log_prob(ts, list(range(len(ts))))       # ratio 1: no token clipped
        before = {n: p.detach().float().cpu().clone() for n, p in w.model.named_parameters()}
        m = w.update_policy(ts)
        after = {n: p.detach().float().cpu() for n, p in w.model.named_parameters()}
        res[dev] = (m, {n: after[n] - before[n] for n in after})
    mc, dc = res["cpu"]
    mg, dg = res["cuda"]
    assert abs(mc["actor/pg_loss"] - mg["actor/pg_loss"]) <= 2e-2 * max(1.0, abs(mc["actor/pg_loss"]))
    assert abs(mc["actor/grad_norm"] - mg["actor/grad_norm"]) <= 5e-2 * mc["actor/grad_norm"]
    # Adam moves every parameter by about lr * sign(grad): the directions agree
    for n in ("layers.0.attn.qkv.weight", "layers.1.mlp.down.weight"):
        agree = (torch.sign(dc[n]) == torch.sign(dg[n])).float().mean().item()
        assert agree > 0.8, (n, agree)
