"""Pipeline parallelism (1F1B over gloo, 2 and 3 stages, with and without
virtual interleaved stages) against the unsplit decoder: every stage's
parameter gradients after a multi-micro-batch step equal the single-rank
gradients of the same parameters, the last stage's losses equal the
single-rank losses, and the forward-only log-probs match."""

import os
import socket
from dataclasses import replace

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _loss(lp, ent, mb):
    return -(lp * mb["w"]).sum() / mb["w"].numel()


def _batches(a, seed=9):
    from psrl_b200.models import packed_positions
    g = torch.Generator().manual_seed(seed)
    out = []
    for lens in ([7, 12], [20], [3, 5, 9], [16, 4], [11]):
        T = sum(lens)
        pos, cu, mx = packed_positions(lens, "cpu")
        out.append({"ids": torch.randint(0, a.vocab_size, (T,), generator=g), "pos": pos, "cu": cu, "max": mx,
                    "labels": torch.randint(0, a.vocab_size, (T,), generator=g), "w": torch.randn(T, generator=g)})
    return out


def _worker(rank, world, port, tied, q, virtual=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.pp import PipelineStage
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a = replace(PRESETS["tiny"], num_layers=max(4, world * virtual), tie_word_embeddings=tied)
    mbs = _batches(a)
    ref = build_model(a, "cpu", torch.float32, seed=2)
    ref_losses = []
    for mb in mbs:
        lp, ent = ref.logprobs(mb["ids"], mb["pos"], mb["cu"], mb["max"], mb["labels"])
        loss = _loss(lp, ent, mb)
        loss.backward()
        ref_losses.append(float(loss))
    ref_grads = {n: p.grad for n, p in ref.named_parameters()}
    stage = PipelineStage(build_model(a, "cpu", torch.float32, seed=2), dist.group.WORLD, virtual=virtual)
    with torch.no_grad():
        ref_lp = [ref.logprobs(mb["ids"], mb["pos"], mb["cu"], mb["max"], mb["labels"])[0] for mb in mbs]
    fwd_err = max(float((y - r).abs().max()) for y, r in zip(stage.forward_only(mbs), ref_lp))
    losses = stage.train_step(mbs, _loss)
    stage.reduce_tied_grads()
    worst, n_params = 0.0, 0
    for n, p in stage.model.named_parameters():
        n_params += 1
        worst = max(worst, float((p.grad - ref_grads[n]).abs().max() / (ref_grads[n].abs().max() + 1e-12)))
    loss_err = max((abs(x - y) for x, y in zip(losses, ref_losses)), default=0.0) if stage.last else 0.0
    q.put({"rank": rank, "grad": worst, "params": n_params, "losses": len(losses), "loss_err": loss_err,
           "layers": (stage.lo, stage.hi), "chunks": stage.chunks, "fwd": fwd_err, "n_layers": a.num_layers})
    dist.destroy_process_group()


@pytest.mark.parametrize("world,tied", [(2, True), (3, False), (3, True)])
def test_pipeline_matches_single_rank(world, tied):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tied, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=600) for _ in range(world)), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    covered = sorted(r["layers"] for r in res)
    assert covered[0][0] == 0 and covered[-1][1] == 4
    for r in res:
        assert r["grad"] < 1e-5, r
    assert res[-1]["losses"] == 5 and res[-1]["loss_err"] < 1e-5
    assert all(r["fwd"] < 1e-5 for r in res), res


@pytest.mark.parametrize("world,virtual,tied", [(2, 2, True), (3, 2, False), (2, 3, False)])
def test_interleaved_pipeline_matches_single_rank(world, virtual, tied):
    """Virtual stages: rank s holds chunks s, s + n, ... of the n x v layer
    chunks; the interleaved schedule (5 micro-batches, not a multiple of n)
    gives the single-rank gradients, losses and forward-only log-probs."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tied, q, virtual)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=600) for _ in range(world)), key=lambda r: r["rank"])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    chunks = sorted(c for r in res for c in r["chunks"])
    assert len(chunks) == world * virtual and chunks[0][0] == 0 and chunks[-1][1] == res[0]["n_layers"]
    assert all(chunks[i][1] == chunks[i + 1][0] for i in range(len(chunks) - 1))
    for r in res:
        assert r["grad"] < 1e-5, r
        assert r["fwd"] < 1e-5, r
    assert res[-1]["losses"] == 5 and res[-1]["loss_err"] < 1e-5


def test_interleaved_timetable_shapes():
    """Every rank runs each (micro-batch, chunk) forward and backward once,
    a backward after its forward, and the bubble shrinks with more chunks."""
    from psrl_b200.parallel.pp import interleaved_timetable
    for n, v, M in ((2, 2, 5), (3, 2, 4), (4, 3, 8), (2, 3, 1), (4, 2, 3)):
        ticks = interleaved_timetable(n, v, M)
        for r in range(n):
            acts = [a[r] for a, _ in ticks if a[r] is not None]
            f = [x[1:] for x in acts if x[0] == "F"]
            b = [x[1:] for x in acts if x[0] == "B"]
            assert sorted(f) == sorted(b) == sorted((k, c) for k in range(M) for c in range(v))
            assert all(acts.index(("F",) + x) < acts.index(("B",) + x) for x in f)
        # every message is received by the rank holding the target chunk
        assert all(dst == g % n for _, msgs in ticks for _, dst, _, _, g in msgs)
    # 4 ranks, 8 micro-batches: 2 chunks per rank need fewer ticks per layer of work
    t1 = len(interleaved_timetable(4, 1, 8)) / 1
    t2 = len(interleaved_timetable(4, 2, 8)) / 2
    assert t2 < t1


def _worker_policy(rank, world, port, q, extra=()):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import copy
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.actor import PolicyWorker
    from psrl_b200.trainer.batch import Trajectory
    init_distributed("cpu", timeout_s=300)
    a = replace(PRESETS["tiny"], num_layers=4)
    # a large Adam eps keeps the update linear in the gradient (see the CP test)
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["actor.optim.lr=1.0", "actor.optim.eps=1.0",
                                                         "actor.ppo_mini_batch_size=4", "actor.ppo_max_token_len_per_gpu=24"]
                      + list(extra))
    g = torch.Generator().manual_seed(4)
    trajs = []
    for i, (P, R) in enumerate(((5, 9), (3, 14), (7, 4), (2, 11))):
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=torch.randint(0, a.vocab_size, (P,), generator=g).tolist(),
                                response_ids=torch.randint(0, a.vocab_size, (R,), generator=g).tolist(),
                                rollout_logprobs=(-torch.rand(R, generator=g)).tolist()))
        trajs[-1].advantage = float(torch.randn(1, generator=g))
    ref = PolicyWorker(cfg, a, "cpu", seed=3)
    ppw = PolicyWorker(cfg, a, "cpu", seed=3, pp_group=dist.group.WORLD)
    t_ref, t_pp = copy.deepcopy(trajs), copy.deepcopy(trajs)
    ref.compute_log_prob(t_ref, list(range(4)))
    ppw.compute_log_prob(t_pp, list(range(4)))
    lp_err = max(abs(x - y) for a_, b_ in zip(t_ref, t_pp) for x, y in zip(a_.old_logprobs, b_.old_logprobs))
    mr = ref.update_policy(t_ref)
    mp_ = ppw.update_policy(t_pp)
    pr, pp_ = dict(ref.model.named_parameters()), dict(ppw.model.named_parameters())
    upd = max(float((pr[n] - pp_[n]).detach().abs().max()) for n in pp_)
    q.put({"rank": rank, "lp": lp_err, "param": upd, "pg": abs(mr["actor/pg_loss"] - mp_["actor/pg_loss"]),
           "owned": len(pp_)})
    dist.destroy_process_group()


@pytest.mark.parametrize("extra", [(), ("actor.virtual_pipeline_parallel_size=2",)])
def test_policy_worker_pipeline_step_matches_single_rank(extra):
    """PolicyWorker with PP=2, plain and with two virtual stages per rank
    (several micro-batches per mini-batch): old log-probs on every stage, the
    loss metric and each stage's parameters after one PPO step equal the
    single-rank worker's."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_policy, args=(r, world, port, q, extra)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in res:
        assert r["lp"] < 1e-4, r
        assert r["param"] < 1e-5, r
        assert r["pg"] < 1e-5, r
