"""Context parallelism (zigzag, CP=2 over gloo) against the unsplit decoder:
the log-probs of every token (gathered back to batch order) and the weight
gradients (summed over the CP ranks) must equal the single-rank ones.  Also a
CPU check of the attention-with-separate-keys reference against the ordinary
causal attention on the same data."""

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
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.parallel.cp import gather_tokens, make_plan, pad_lengths
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a = PRESETS["tiny"]
    model = build_model(a, "cpu", torch.float32, seed=5)
    lens = pad_lengths([13, 29, 6], world)                    # 16, 32, 8
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, a.vocab_size, (sum(lens),), generator=g)
    labels = torch.randint(0, a.vocab_size, (sum(lens),), generator=g)
    wts = torch.randn(sum(lens), generator=g)
    pos, cu, mx = packed_positions(lens, "cpu")
    # reference: the whole batch on one rank
    lp_full, _ = model.logprobs(ids, pos, cu, mx, labels)
    (lp_full * wts).sum().backward()
    ref_grads = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    # context parallel: this rank's zigzag share
    plan = make_plan(lens, dist.group.WORLD)
    li = plan.local_idx
    lp_loc, _ = model.logprobs(ids[li], pos[li], plan, plan.max_q, labels[li])
    (lp_loc * wts[li]).sum().backward()
    worst = 0.0
    for n, p in model.named_parameters():
        gsum = p.grad.clone()
        dist.all_reduce(gsum)
        worst = max(worst, float((gsum - ref_grads[n]).abs().max() / (ref_grads[n].abs().max() + 1e-12)))
    lp_all = gather_tokens(lp_loc.detach(), plan)
    q.put({"rank": rank, "lp": float((lp_all - lp_full.detach()).abs().max()), "grad": worst,
           "local": plan.num_local, "total": sum(lens)})
    dist.destroy_process_group()


def test_context_parallel_matches_single_rank():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in res:
        assert r["local"] * world == r["total"]
        assert r["lp"] < 1e-4, r
        assert r["grad"] < 1e-4, r


def test_zigzag_rows_cover_the_batch_once():
    from psrl_b200.parallel.cp import zigzag_rows
    lens = [8, 16, 24]
    rows = [zigzag_rows(lens, 4, r) for r in range(4)]
    flat = sorted(i for rr in rows for i in rr)
    assert flat == list(range(sum(lens)))
    # rank 0 of the first sequence: chunks 0 and 7 (one token each)
    assert rows[0][:2] == [0, 7]


def test_attention_kv_ref_equals_causal_suffix():
    from psrl_b200.ops.attention import attention_kv_ref, varlen_attention_ref
    torch.manual_seed(0)
    nq, nkv, d, L = 4, 2, 16, 20
    q = torch.randn(L, nq, d)
    k = torch.randn(L, nkv, d)
    v = torch.randn(L, nkv, d)
    full = varlen_attention_ref(q, k, v, torch.tensor([0, L], dtype=torch.int32), 0.25)
    # queries 12..19 against keys 0..19 are the last 8 of 20 positions
    part = attention_kv_ref(q[12:], k, v, torch.tensor([0, 8], dtype=torch.int32),
                            torch.tensor([0, L], dtype=torch.int32), 0.25)
    torch.testing.assert_close(part, full[12:])


def _worker_policy(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.actor import PolicyWorker
    from psrl_b200.trainer.batch import Trajectory
    init_distributed("cpu", timeout_s=300)
    a = PRESETS["tiny"]
    # a large Adam eps makes the update linear in the gradient, so the check sees
    # gradient differences instead of the sign of near-zero gradients
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["actor.optim.lr=1.0", "actor.optim.eps=1.0",
                                                         "actor.ppo_mini_batch_size=4"])
    g = torch.Generator().manual_seed(4)
    trajs = []
    for i, (P, R) in enumerate(((5, 9), (3, 14), (7, 4), (2, 11))):
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=torch.randint(0, a.vocab_size, (P,), generator=g).tolist(),
                                response_ids=torch.randint(0, a.vocab_size, (R,), generator=g).tolist(),
                                rollout_logprobs=(-torch.rand(R, generator=g)).tolist()))
        trajs[-1].advantage = float(torch.randn(1, generator=g))
    ref = PolicyWorker(cfg, a, "cpu", seed=3)                                       # one rank, whole sequences
    cpw = PolicyWorker(cfg, a, "cpu", seed=3, dp_group=dist.group.WORLD, cp_group=dist.group.WORLD)
    import copy
    t_ref, t_cp = copy.deepcopy(trajs), copy.deepcopy(trajs)
    ref.compute_log_prob(t_ref, list(range(4)))
    cpw.compute_log_prob(t_cp, list(range(4)))
    lp_err = max(abs(x - y) for a_, b_ in zip(t_ref, t_cp) for x, y in zip(a_.old_logprobs, b_.old_logprobs))
    ref.update_policy(t_ref)
    cpw.update_policy(t_cp)
    pr, pc = dict(ref.model.named_parameters()), dict(cpw.model.named_parameters())
    upd = max(float((pr[n] - pc[n]).detach().abs().max()) for n in pr)
    q.put({"rank": rank, "lp": lp_err, "param": upd})
    dist.destroy_process_group()


def test_policy_worker_context_parallel_step_matches_single_rank():
    """PolicyWorker with CP=2: old log-probs and the parameters after one PPO
    step equal those of the single-rank worker on the same trajectories."""
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
