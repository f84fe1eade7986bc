"""Tensor parallelism (TP=2 over gloo) against the unsharded decoder: forward
outputs, gradients, and one optimizer step of the TP PolicyWorker, which must
leave every shard equal to the matching slice of the unsharded model's update."""

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS, packed_positions
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.actor import PolicyWorker
    init_distributed("cpu", timeout_s=300)
    a = PRESETS["tiny"]
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["actor.optim.lr=1e-2"])
    ref = PolicyWorker(cfg, a, "cpu", seed=3)                                     # unsharded, single rank
    tpw = PolicyWorker(cfg, a, "cpu", seed=3, tp_group=dist.group.WORLD)         # TP=2, DP=1
    g = torch.Generator().manual_seed(7)                                          # same data on both TP ranks
    lens = [19, 33, 8]
    ids = torch.randint(0, a.vocab_size, (sum(lens),), generator=g)
    pos, cu, mx = packed_positions(lens, "cpu")
    coef = torch.randn(sum(lens), a.hidden_size, generator=g)
    out = {"rank": rank}
    hr = ref.model.hidden_states(ids, pos, cu, mx)
    ht = tpw.model.hidden_states(ids, pos, cu, mx)
    out["fwd"] = float((hr - ht).detach().abs().max() / hr.detach().abs().max())
    (hr * coef).sum().backward()
    (ht * coef).sum().backward()
    # the main-grad buffers hold the gradients before the step; compare the down projection's
    gref = ref.dp.flat_grad.clone()
    l0 = ref.model.layers[0].mlp.down.weight
    il = a.intermediate_size // 2
    b0, off0 = ref.dp.param_to_bucket[l0]
    g_full = b0.grad[off0: off0 + l0.numel()].view(l0.shape)[:, rank * il:(rank + 1) * il]
    mine = tpw.model.layers[0].mlp.down_weight
    b1, off1 = tpw.dp_partner.param_to_bucket[mine]
    g_tp = b1.grad[off1: off1 + mine.numel()].view(mine.shape)
    out["grad"] = float((g_full - g_tp).abs().max() / g_full.abs().max())
    del gref
    sr = ref.dp.step()
    st = tpw.dp.step(partners=[tpw.dp_partner])
    out["norm"] = (float(sr["grad_norm"]), float(st["grad_norm"]))
    # compare updated parameters: TP shard vs the slice of the unsharded update
    d, r, P = a.head_dim, rank, 2
    qn, kn = a.num_heads // P * d, a.num_kv_heads // P * d
    worst = 0.0
    for i in range(a.num_layers):
        full = ref.model.layers[i]
        mine = tpw.model.layers[i]
        w = full.attn.qkv.weight
        rows = torch.cat([torch.arange(r * qn, (r + 1) * qn), a.q_size + torch.arange(r * kn, (r + 1) * kn),
                          a.q_size + a.kv_size + torch.arange(r * kn, (r + 1) * kn)])
        pairs = [(w[rows], mine.attn.qkv_weight), (full.attn.o.weight[:, r * qn:(r + 1) * qn], mine.attn.o_weight)]
        il = a.intermediate_size // P
        gu = full.mlp.gate_up.weight
        pairs.append((torch.cat([gu[r * il:(r + 1) * il], gu[a.intermediate_size + r * il:
                                                             a.intermediate_size + (r + 1) * il]]),
                      mine.mlp.gate_up_weight))
        pairs.append((full.mlp.down.weight[:, r * il:(r + 1) * il], mine.mlp.down_weight))
        pairs.append((full.ln1, mine.ln1))
        for x, y in pairs:
            worst = max(worst, float((x.detach() - y.detach()).abs().max()))
    worst = max(worst, float((ref.model.embed.weight - tpw.model.embed.weight).detach().abs().max()))
    out["param_diff"] = worst
    q.put(out)
    dist.destroy_process_group()


def test_tensor_parallel_matches_unsharded_decoder():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    for r in [q.get(timeout=5) for _ in range(2)]:
        assert r["fwd"] < 1e-5, r
        nr, nt = r["norm"]
        assert abs(nr - nt) < 1e-4 * max(1.0, nr), r
        assert r["grad"] < 1e-5, r
        # Adam's first step is sign-like (lr = 1e-2 per element): near-zero gradients
        # that differ in the last bits may move differently, never by a whole step
        assert r["param_diff"] < 1e-3, r


def _assemble_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.assemble import FullWeightAssembler
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.rollout.engine import EngineWeights
    from psrl_b200.trainer.actor import PolicyWorker
    init_distributed("cpu", timeout_s=300)
    worst = {}
    for label, preset, kw, ep in (
            ("tiny", "tiny", {"tp_group": dist.group.WORLD}, 2),
            ("tiny-moe", "tiny-moe", {"dp_group": dist.group.WORLD, "dp_rank": rank, "dp_world": world}, 2),
            ("tiny-moe-tp", "tiny-moe", {"tp_group": dist.group.WORLD}, 1)):
        a = PRESETS[preset]
        cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"model.preset={preset}",
                                                             f"++actor.expert_parallel_size={ep}"])
        w = PolicyWorker(cfg, a, "cpu", seed=9, **kw)
        asm = FullWeightAssembler(w.model, ep=w.ep, tp=w.tp,
                                  ep_names=[n for n, _ in w.model.named_parameters() if "experts_w" in n]
                                  if w.ep is not None else (),
                                  tp_names=sorted(w.tp_sharded) if w.tp is not None else ())
        eng = EngineWeights.from_model(build_model(a, "cpu", torch.float32, seed=123), "cpu", torch.float32)
        asm.gather()
        asm.assemble_into(eng.tensors)
        ref = dict(build_model(a, "cpu", torch.float32, seed=9).named_parameters())
        worst[label] = max(float((eng.tensors[n] - p.detach()).abs().max()) for n, p in ref.items())
    q.put(worst)
    dist.destroy_process_group()


def test_full_weight_assembly_from_tp_and_ep_shards():
    """The rollout engine's full weights assembled from TP / EP shards (and
    from tensor-parallel experts) equal the unsharded model's weights exactly."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_assemble_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    assert [p.exitcode for p in procs] == [0, 0]
    for _ in range(2):
        w = q.get(timeout=5)
        assert w["tiny"] == 0.0 and w["tiny-moe"] == 0.0 and w["tiny-moe-tp"] == 0.0, w


def _engine_worker(rank, world, port, q, preset="tiny", shared=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.parallel.tp import make_tp_group, shard_engine_tensors
    from psrl_b200.rollout.engine import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    init_distributed("cpu", timeout_s=300)
    from dataclasses import replace
    a = PRESETS[preset]
    if shared:
        a = replace(a, shared_expert_intermediate_size=shared)
    full = EngineWeights.from_model(build_model(a, "cpu", torch.float32, seed=4), "cpu", torch.float32)
    tp = make_tp_group(dist.group.WORLD)
    shard = EngineWeights(a, "cpu", torch.float32)
    shard.tensors = shard_engine_tensors(a, full.tensors, tp)

    def run(w, tpg):
        eng = RolloutEngine(a, w, max_num_seqs=4, max_model_len=128, block_size=16, kv_cache_gb=0.05,
                            use_cuda_graph=False, enable_prefix_caching=False, tp=tpg)
        for i in range(3):
            eng.add_request(GenRequest(i, list(range(5, 20 + 3 * i)), SamplingParams(temperature=0.0, max_tokens=10,
                                                                                     ignore_eos=True, seed=i)))
        outs = {}
        while eng.has_unfinished():
            for o in eng.step():
                outs[o.request_id] = (list(o.output_ids), list(o.logprobs))
        return outs

    ref = run(full, None)
    got = run(shard, tp)
    same = all(ref[i][0] == got[i][0] for i in ref)
    lp = max(abs(x - y) for i in ref for x, y in zip(ref[i][1], got[i][1]))
    q.put({"rank": rank, "same_tokens": same, "lp_diff": lp})
    dist.destroy_process_group()


@pytest.mark.parametrize("preset,shared,world", [("tiny", 0, 2), ("tiny-moe", 0, 2), ("tiny-moe", 128, 2),
                                                 ("tiny", 0, 4)])
def test_tensor_parallel_rollout_engine_matches_single_rank(preset, shared, world):
    """A TP rollout engine (gloo ranks, identical request streams) decodes the
    same greedy tokens and log-probs as the unsharded engine; for MoE the
    experts are split over the ranks (expert parallelism follows TP), with and
    without a TP-sharded shared expert; at TP=4 over 2 KV heads each KV head
    is replicated on the two ranks whose query heads read it."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_engine_worker, args=(r, world, port, q, preset, shared)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    assert [p.exitcode for p in procs] == [0] * world
    for _ in range(world):
        r = q.get(timeout=5)
        assert r["same_tokens"], r
        assert r["lp_diff"] < 1e-4, r


def _ckpt_worker(rank, world, port, q, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.models.hf_io import load_hf_into
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.actor import PolicyWorker
    from psrl_b200.utils.checkpoint import load_worker, save_worker
    init_distributed("cpu", timeout_s=300)
    out = {"rank": rank}
    for label, preset, kw, ep in (
            ("tiny", "tiny", {"tp_group": dist.group.WORLD}, 2),
            ("tiny-moe", "tiny-moe", {"dp_group": dist.group.WORLD, "dp_rank": rank, "dp_world": world}, 2),
            ("tiny-moe-tp", "tiny-moe", {"tp_group": dist.group.WORLD}, 1)):
        a = PRESETS[preset]
        cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"model.preset={preset}",
                                                             f"++actor.expert_parallel_size={ep}"])
        d = os.path.join(path, label)
        w = PolicyWorker(cfg, a, "cpu", seed=21, **kw)
        save_worker(w, d, rank)
        dist.barrier()
        # the HF export is the unsharded model
        full = build_model(a, "cpu", torch.float32, seed=0)
        load_hf_into(full, d)
        ref = build_model(a, "cpu", torch.float32, seed=21)
        rp = dict(ref.named_parameters())
        out[label + "_hf"] = max(float((p.detach() - rp[n].detach()).abs().max()) for n, p in full.named_parameters())
        # a differently initialised sharded worker reloads the same shards
        w2 = PolicyWorker(cfg, a, "cpu", seed=99, **kw)
        load_worker(w2, d, rank)
        p1 = dict(w.model.named_parameters())
        out[label + "_reload"] = max(float((p.detach() - p1[n].detach()).abs().max())
                                      for n, p in w2.model.named_parameters())
    q.put(out)
    dist.destroy_process_group()


def test_sharded_worker_checkpoint_roundtrip(tmp_path):
    """TP and EP workers export the full model in HF format and reload their shards."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ckpt_worker, args=(r, 2, port, q, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    assert [p.exitcode for p in procs] == [0, 0]
    for _ in range(2):
        r = q.get(timeout=5)
        for k in ("tiny_hf", "tiny_reload", "tiny-moe_hf", "tiny-moe_reload", "tiny-moe-tp_hf", "tiny-moe-tp_reload"):
            assert r[k] == 0.0, r


def _etp_worker(rank, world, port, q, shared):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from dataclasses import replace
    import torch
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS, packed_positions
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.actor import PolicyWorker
    init_distributed("cpu", timeout_s=300)
    a = replace(PRESETS["tiny-moe"], shared_expert_intermediate_size=shared)
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["model.preset=tiny-moe", "actor.optim.lr=1e-2",
                                                         "actor.optim.eps=1.0"])
    ref = PolicyWorker(cfg, a, "cpu", seed=3)
    tpw = PolicyWorker(cfg, a, "cpu", seed=3, tp_group=dist.group.WORLD)
    g = torch.Generator().manual_seed(7)
    lens = [11, 17, 6]
    ids = torch.randint(0, a.vocab_size, (sum(lens),), generator=g)
    pos, cu, mx = packed_positions(lens, "cpu")
    coef = torch.randn(sum(lens), a.hidden_size, generator=g)
    out = {"rank": rank}
    hr = ref.model.hidden_states(ids, pos, cu, mx)
    ht = tpw.model.hidden_states(ids, pos, cu, mx)
    out["fwd"] = float((hr - ht).detach().abs().max() / hr.detach().abs().max())
    (hr * coef).sum().backward()
    (ht * coef).sum().backward()

    def grad(dp, p):
        b, off = dp.param_to_bucket[p]
        return b.grad[off: off + p.numel()].view(p.shape)

    I, il = a.moe_intermediate_size, a.moe_intermediate_size // 2
    m_ref, m_tp = ref.model.layers[0].mlp, tpw.model.layers[0].mlp
    g_w2 = grad(ref.dp, m_ref.experts_w2)[:, :, rank * il:(rank + 1) * il]
    g_w13 = grad(ref.dp, m_ref.experts_w13)
    g_w13 = torch.cat([g_w13[:, rank * il:(rank + 1) * il], g_w13[:, I + rank * il:I + (rank + 1) * il]], dim=1)
    errs = [float((g_w2 - grad(tpw.dp_partner, m_tp.experts_w2)).abs().max() / g_w2.abs().max()),
            float((g_w13 - grad(tpw.dp_partner, m_tp.experts_w13)).abs().max() / g_w13.abs().max())]
    # replicated router: the summed partial gradients equal the unsharded gradient
    g_r = grad(ref.dp, m_ref.router.weight)
    errs.append(float((g_r - grad(tpw.dp, m_tp.router.weight)).abs().max() / g_r.abs().max()))
    if shared:
        g_s = grad(ref.dp, m_ref.shared_gate.weight)
        errs.append(float((g_s - grad(tpw.dp, m_tp.shared_gate.weight)).abs().max() / g_s.abs().max()))
    out["grad"] = max(errs)
    sr = ref.dp.step()
    st = tpw.dp.step(partners=[tpw.dp_partner])
    out["norm"] = (float(sr["grad_norm"]), float(st["grad_norm"]))
    w2_new = m_ref.experts_w2[:, :, rank * il:(rank + 1) * il]
    out["param_diff"] = max(float((w2_new - m_tp.experts_w2).detach().abs().max()),
                            float((m_ref.router.weight - m_tp.router.weight).detach().abs().max()))
    q.put(out)
    dist.destroy_process_group()


@pytest.mark.parametrize("shared", [0, 128])
def test_expert_tensor_parallel_matches_unsharded_moe(shared):
    """TP=2 on a MoE decoder (each expert's width split, router replicated, its
    partial gradients summed over the group): forward, gradients, grad norm
    and the updated parameters equal the unsharded worker's, with and without
    a shared expert."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_etp_worker, args=(r, 2, port, q, shared)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    assert [p.exitcode for p in procs] == [0, 0]
    for r in [q.get(timeout=5) for _ in range(2)]:
        assert r["fwd"] < 1e-5, r
        assert r["grad"] < 1e-5, r
        nr, nt = r["norm"]
        assert abs(nr - nt) < 1e-4 * max(1.0, nr), r
        assert r["param_diff"] < 1e-5, r
