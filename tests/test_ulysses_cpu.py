"""Ulysses sequence parallelism (2 gloo ranks) against the unsplit decoder:
log-probs gathered back to batch order and weight gradients summed over the
ranks equal the single-rank ones, also when the token count needs padding;
a PolicyWorker step with ``cp_mode="ulysses"`` equals the single-rank step."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, lens):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.parallel.ulysses import UlyssesShard
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a = PRESETS["tiny"]                      # 4 query / 2 KV heads
    model = build_model(a, "cpu", torch.float32, seed=5)
    g = torch.Generator().manual_seed(11)
    T = sum(lens)
    ids = torch.randint(0, a.vocab_size, (T,), generator=g)
    labels = torch.randint(0, a.vocab_size, (T,), generator=g)
    wts = torch.randn(T, generator=g)
    pos, cu, mx = packed_positions(lens, "cpu")
    lp_full, _ = model.logprobs(ids, pos, cu, mx, labels)
    (lp_full * wts).sum().backward()
    ref_grads = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    sh = UlyssesShard(cu, dist.group.WORLD)
    lp_loc, _ = model.logprobs(sh.local(ids), sh.positions(), sh.plan, sh.plan.max_q, sh.local(labels))
    (lp_loc * sh.local(wts, 0.0)).sum().backward()
    worst = 0.0
    for n, p in model.named_parameters():
        gsum = p.grad.clone()
        dist.all_reduce(gsum)
        worst = max(worst, float((gsum - ref_grads[n]).abs().max() / (ref_grads[n].abs().max() + 1e-12)))
    lp_all = sh.full(lp_loc.detach())
    q.put({"rank": rank, "lp": float((lp_all - lp_full.detach()).abs().max()), "grad": worst})
    dist.destroy_process_group()


@pytest.mark.parametrize("lens", [[13, 29, 6], [7, 20]])     # 48 tokens; 27 tokens (one padding row)
def test_ulysses_matches_single_rank(lens):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, lens)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in res:
        assert r["lp"] < 1e-5, r
        assert r["grad"] < 1e-5, r


def _worker_policy(rank, world, port, q):
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
    a = PRESETS["tiny"]
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["actor.optim.lr=1.0", "actor.optim.eps=1.0",
                                                         "actor.ppo_mini_batch_size=4"])
    g = torch.Generator().manual_seed(4)
    trajs = []
    for i, (P, R) in enumerate(((5, 9), (3, 14), (7, 4), (2, 11))):
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=torch.randint(0, a.vocab_size, (P,), generator=g).tolist(),
                                response_ids=torch.randint(0, a.vocab_size, (R,), generator=g).tolist(),
                                rollout_logprobs=(-torch.rand(R, generator=g)).tolist()))
        trajs[-1].advantage = float(torch.randn(1, generator=g))
    ref = PolicyWorker(cfg, a, "cpu", seed=3)
    # both ranks hold every sequence (data parallelism 1) and split each micro-batch
    usp = PolicyWorker(cfg, a, "cpu", seed=3, dp_group=dist.group.WORLD, cp_group=dist.group.WORLD,
                       cp_mode="ulysses")
    t_ref, t_sp = copy.deepcopy(trajs), copy.deepcopy(trajs)
    ref.compute_log_prob(t_ref, list(range(4)))
    usp.compute_log_prob(t_sp, list(range(4)))
    lp = max(abs(x - y) for a_, b_ in zip(t_ref, t_sp) for x, y in zip(a_.old_logprobs, b_.old_logprobs))
    mr = ref.update_policy(t_ref)
    ms = usp.update_policy(t_sp)
    pr, ps = dict(ref.model.named_parameters()), dict(usp.model.named_parameters())
    # each rank reports its tokens' share of the token-normalised loss
    pg = torch.tensor([ms["actor/pg_loss"]], dtype=torch.float64)
    dist.all_reduce(pg)
    q.put({"rank": rank, "lp": lp, "param": max(float((pr[n] - ps[n]).detach().abs().max()) for n in ps),
           "pg": abs(mr["actor/pg_loss"] - float(pg))})
    dist.destroy_process_group()


def test_policy_worker_ulysses_step_matches_single_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_policy, args=(r, world, port, q)) for r in range(world)]
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
