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
    # a small token budget: ranks pack different numbers of micro-batches, which
    # gradient sharding must pad to the same count (its backward is collective)
    base = ["actor.optim.lr=1.0", "actor.optim.eps=1.0", "actor.ppo_mini_batch_size=8",
            "actor.ppo_max_token_len_per_gpu=20"]
    g = torch.Generator().manual_seed(4)
    trajs = []
    for i in range(8):
        P, R = 3 + i % 4, 5 + (3 * i) % 7 if i % 4 else 2
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=torch.randint(0, a.vocab_size, (P,), generator=g).tolist(),
                                response_ids=torch.randint(0, a.vocab_size, (R,), generator=g).tolist(),
                                rollout_logprobs=(-torch.rand(R, generator=g)).tolist()))
        trajs[-1].advantage = float(torch.randn(1, generator=g))
    out = {}
    for name, extra in (("full", []), ("hsdp", ["actor.fsdp_size=2", "actor.fsdp_shard_grads=true"])):
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
    """PolicyWorker with actor.fsdp_size=2 and gradient sharding on 4 ranks:
    the PPO step leaves the same parameters as sharding over all 4 ranks with
    full gradient buffers."""
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


def _worker_shard_grads(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.parallel.fsdp import FlatShardedDP, hybrid_shard_groups
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a = PRESETS["tiny"]
    shard, rep = hybrid_shard_groups(dist.group.WORLD, 2)
    kw = dict(lr=1e-2, eps=1.0, weight_decay=0.1, max_grad_norm=1.0)
    runs = {}
    for name, extra in (("full", dict(group=dist.group.WORLD)),
                        ("sharded", dict(group=dist.group.WORLD, shard_grads=True)),
                        ("hsdp_sharded", dict(group=shard, replicate_group=rep, shard_grads=True))):
        model = build_model(a, "cpu", torch.float32, seed=1)
        dp = FlatShardedDP(model, extra.pop("group"), **extra, **kw)
        g = torch.Generator().manual_seed(70 + rank)
        norms = []
        for _ in range(2):                       # optimizer steps
            for lens in ([5, 9], [12], [3, 4, 6]):   # micro-batches
                T = sum(lens)
                pos, cu, mx = packed_positions(lens, "cpu")
                ids = torch.randint(0, a.vocab_size, (T,), generator=g)
                lab = torch.randint(0, a.vocab_size, (T,), generator=g)
                lp, _ = model.logprobs(ids, pos, cu, mx, lab)
                (-lp.mean()).backward()
            norms.append(float(dp.step()["grad_norm"]))
        runs[name] = (dp, norms)
    base = runs["full"][0].flat
    out = {"rank": rank, "grad_buffer": runs["sharded"][0].flat_grad.numel()}
    for name in ("sharded", "hsdp_sharded"):
        out[name] = (float((runs[name][0].flat - base).abs().max()),
                     max(abs(x - y) for x, y in zip(runs[name][1], runs["full"][1])))
    q.put(out)
    dist.destroy_process_group()


def test_gradient_sharding_matches_full_gradients():
    """shard_grads=True (no model-wide fp32 gradient buffer; each layer bucket
    reduce-scattered as its backward completes), alone and with hybrid
    sharding: same gradient norms and parameters as the full-buffer path
    after two steps of three micro-batches each."""
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_shard_grads, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in res:
        assert r["grad_buffer"] == 0, r
        for name in ("sharded", "hsdp_sharded"):
            assert r[name][0] < 1e-6 and r[name][1] < 1e-4, (name, r)
