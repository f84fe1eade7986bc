"""Hybrid sharding (HSDP) of the sharded optimizer: 4 gloo ranks as 2 shard
groups x 2 replicas take the same step as plain sharding over all 4 ranks
(the gradients are summed over every rank either way), and every rank ends
with the same parameters."""

import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.fsdp import FlatShardedDP, hybrid_shard_groups
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a = PRESETS["tiny"]
    shard, rep = hybrid_shard_groups(dist.group.WORLD, 2)
    # a large Adam eps keeps the update linear in the gradient, so the two
    # summation orders differ only by fp32 rounding
    kw = dict(lr=1e-2, eps=1.0, weight_decay=0.1, max_grad_norm=1.0)
    full = FlatShardedDP(build_model(a, "cpu", torch.float32, seed=1), dist.group.WORLD, **kw)
    hyb = FlatShardedDP(build_model(a, "cpu", torch.float32, seed=1), shard, replicate_group=rep, **kw)
    g = torch.Generator().manual_seed(50 + rank)
    norms = []
    for _ in range(3):
        grad = torch.randn(full.total, generator=g) * 0.05
        full.flat_grad.copy_(grad)
        hyb.flat_grad.copy_(grad)
        norms.append((float(full.step()["grad_norm"]), float(hyb.step()["grad_norm"])))
    diff = float((full.flat - hyb.flat).abs().max())
    same = hyb.flat.clone()
    dist.all_reduce(same, op=dist.ReduceOp.MAX)
    q.put({"rank": rank, "diff": diff, "norms": norms, "same": bool(torch.equal(same, hyb.flat)),
           "shard_world": hyb.world})
    dist.destroy_process_group()


def test_hybrid_sharding_matches_full_sharding():
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in res:
        assert r["shard_world"] == 2
        assert r["diff"] < 1e-6, r
        assert r["same"], r
        assert all(abs(x - y) < 1e-5 * max(1.0, x) for x, y in r["norms"]), r


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
    base = ["actor.optim.lr=1.0", "actor.optim.eps=1.0", "actor.ppo_mini_batch_size=8"]
    g = torch.Generator().manual_seed(4)
    trajs = []
    for i in range(8):
        P, R = 3 + i % 4, 5 + (3 * i) % 7
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=torch.randint(0, a.vocab_size, (P,), generator=g).tolist(),
                                response_ids=torch.randint(0, a.vocab_size, (R,), generator=g).tolist(),
                                rollout_logprobs=(-torch.rand(R, generator=g)).tolist()))
        trajs[-1].advantage = float(torch.randn(1, generator=g))
    out = {}
    for name, extra in (("full", []), ("hsdp", ["actor.fsdp_size=2"])):
        cfg = load_config(preset="cpu_tiny_grpo", overrides=base + extra)
        w = PolicyWorker(cfg, a, "cpu", seed=3, dp_group=dist.group.WORLD, dp_rank=rank, dp_world=world)
        t = copy.deepcopy(trajs)
        w.compute_log_prob(t, list(range(len(t))))
        w.update_policy(t)
        out[name] = (w, w.dp.world)
    pf, ph = dict(out["full"][0].model.named_parameters()), dict(out["hsdp"][0].model.named_parameters())
    diff = max(float((pf[n] - ph[n]).detach().abs().max()) for n in pf)
    q.put({"rank": rank, "diff": diff, "shard_world": out["hsdp"][1], "full_world": out["full"][1]})
    dist.destroy_process_group()


def test_policy_worker_hybrid_sharding_step():
    """PolicyWorker with actor.fsdp_size=2 on 4 ranks: the PPO step leaves the
    same parameters as sharding over all 4 ranks."""
    world = 4
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
        assert r["shard_world"] == 2 and r["full_world"] == 4, r
        assert r["diff"] < 1e-5, r
