"""Context parallelism on 2 GPUs (NCCL all-gather of keys / values,
reduce-scatter of their gradients, tcgen05 attention of query chunks against
key prefixes) against the unsplit bf16 decoder on one GPU."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.parallel.cp import gather_tokens, make_plan, pad_lengths
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", rank)
    a = PRESETS["tiny128"]
    model = build_model(a, dev, torch.bfloat16, seed=5)
    lens = pad_lengths([700, 1290, 100], world)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, a.vocab_size, (sum(lens),), generator=g).to(dev)
    labels = torch.randint(0, a.vocab_size, (sum(lens),), generator=g).to(dev)
    wts = torch.randn(sum(lens), generator=g).to(dev)
    pos, cu, mx = packed_positions(lens, dev)
    lp_full, _ = model.logprobs(ids, pos, cu, mx, labels)
    (lp_full * wts).sum().backward()
    ref = {n: p.grad.float().clone() for n, p in model.named_parameters()}
    model.zero_grad(set_to_none=True)
    plan = make_plan(lens, dist.group.WORLD, dev)
    li = plan.local_idx
    lp_loc, _ = model.logprobs(ids[li], pos[li], plan, plan.max_q, labels[li])
    (lp_loc * wts[li]).sum().backward()
    torch.cuda.synchronize()
    check_errors()
    worst = 0.0
    for n, p in model.named_parameters():
        gs = p.grad.float().clone()
        dist.all_reduce(gs)
        worst = max(worst, float((gs - ref[n]).abs().max() / (ref[n].abs().max() + 1e-6)))
    lp_all = gather_tokens(lp_loc.detach(), plan)
    q.put({"rank": rank, "lp": float((lp_all - lp_full.detach()).abs().max()), "grad": worst})
    dist.destroy_process_group()


def test_context_parallel_two_gpus_matches_one():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in res:
        assert r["lp"] < 5e-2, r          # bf16 log-probs of the same tokens
        assert r["grad"] < 5e-2, r        # relative to each gradient's largest entry
