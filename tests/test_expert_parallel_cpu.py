"""Expert parallelism on two gloo ranks against the unsharded MoE model:
forward outputs, gradients of the dense parameters and of each rank's experts,
and one optimizer step of the expert-parallel PolicyWorker."""

import os
import socket

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
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.parallel.ep import make_ep_group, shard_experts
    init_distributed("cpu", timeout_s=300)
    a = PRESETS["tiny-moe"]
    ref = build_model(a, "cpu", torch.float32, seed=5)
    epm = build_model(a, "cpu", torch.float32, seed=5)
    ep = make_ep_group(dist.group.WORLD, a.num_experts)
    names = shard_experts(epm, ep)
    g = torch.Generator().manual_seed(rank)
    lens = [23, 41] if rank == 0 else [17, 9, 30]
    ids = torch.randint(0, a.vocab_size, (sum(lens),), generator=g)
    pos, cu, mx = packed_positions(lens, "cpu")
    coef = torch.randn(sum(lens), a.hidden_size, generator=g)
    out = {"rank": rank}
    h_ref = ref.hidden_states(ids, pos, cu, mx)
    h_ep = epm.hidden_states(ids, pos, cu, mx)
    out["fwd"] = float((h_ref - h_ep).detach().abs().max())
    (h_ref * coef).sum().backward()
    (h_ep * coef).sum().backward()
    # dense grads: per-rank equal; expert grads: EP rank holds the sum over both ranks' tokens
    dense = max(float((p.grad - dict(epm.named_parameters())[n].grad).abs().max() / (p.grad.abs().max() + 1e-12))
                for n, p in ref.named_parameters() if n not in names and p.grad is not None)
    out["dense_grad"] = dense
    worst = 0.0
    rp = dict(ref.named_parameters())
    for n in names:
        full = rp[n].grad.clone()
        dist.all_reduce(full)
        mine = full[ep.first: ep.first + ep.local]
        worst = max(worst, float((mine - dict(epm.named_parameters())[n].grad).abs().max() /
                                 (mine.abs().max() + 1e-12)))
    out["expert_grad_rel"] = worst
    # one expert-parallel optimizer step through PolicyWorker
    from psrl_b200.config import load_config
    from psrl_b200.trainer.actor import PolicyWorker
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["model.preset=tiny-moe", "++actor.expert_parallel_size=2"])
    w = PolicyWorker(cfg, a, "cpu", dp_group=dist.group.WORLD, seed=5, dp_rank=rank, dp_world=world)
    h = w.model.hidden_states(ids, pos, cu, mx)
    (h * coef).sum().backward()
    before = w.model.layers[0].mlp.experts_w13.detach().clone()
    st = w.dp.step(partners=[w.dp_partner])
    out["moved"] = float((w.model.layers[0].mlp.experts_w13.detach() - before).abs().max())
    out["grad_norm"] = float(st["grad_norm"])
    q.put(out)
    dist.destroy_process_group()


def test_expert_parallel_matches_unsharded_moe():
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
    res = sorted([q.get(timeout=5) for _ in range(2)], key=lambda d: d["rank"])
    for r in res:
        assert r["fwd"] < 1e-4, r
        assert r["dense_grad"] < 1e-4, r      # relative to each parameter's largest gradient
        assert r["expert_grad_rel"] < 1e-4, r
        assert r["moved"] > 0, r
    assert abs(res[0]["grad_norm"] - res[1]["grad_norm"]) < 1e-6 * max(1.0, res[0]["grad_norm"])
