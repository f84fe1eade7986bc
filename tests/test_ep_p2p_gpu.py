"""Expert-parallel all-to-all over NVLink peer memory on 2 GPUs against
NCCL's all_to_all_single (ragged, empty and skewed splits, forward and the
transposed backward), and an expert-parallel MoE layer (forward + backward)
with the peer path against the NCCL path."""

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
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.parallel.ep import make_ep_group, moe_forward_ep
    from psrl_b200.parallel.ep_p2p import PeerAllToAll, peer_all_to_all
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", rank)
    a2a = PeerAllToAll(dist.group.WORLD, dev, 64 << 20)
    res = {"rank": rank}
    worst = 0.0
    for case, send in enumerate(([3, 5], [0, 7], [1000, 1], [0, 0], [257, 513])):
        g = torch.Generator(device=dev).manual_seed(case * 10 + rank)
        x = torch.randn(sum(send), 128, device=dev, generator=g).bfloat16().requires_grad_(True)
        M = a2a.counts(send)
        y = peer_all_to_all(x, M, a2a)
        recv = [M[s][rank] for s in range(world)]
        ref = torch.empty(sum(recv), 128, dtype=x.dtype, device=dev)
        dist.all_to_all_single(ref, x.detach().contiguous(), recv, send)
        worst = max(worst, float((y.float() - ref.float()).abs().max()) if ref.numel() else 0.0)
        gy = torch.randn_like(y)
        y.backward(gy)
        gref = torch.empty_like(x)
        dist.all_to_all_single(gref, gy.contiguous(), send, recv)
        worst = max(worst, float((x.grad.float() - gref.float()).abs().max()) if x.numel() else 0.0)
    res["a2a"] = worst
    # a MoE layer: peer path vs NCCL path on the same data
    E, h, I, T, k = 8, 256, 128, 300, 2
    gen = torch.Generator(device=dev).manual_seed(7)          # same experts everywhere, then sliced
    w13 = (torch.randn(E, 2 * I, h, device=dev, generator=gen) * 0.05).bfloat16()
    w2 = (torch.randn(E, h, I, device=dev, generator=gen) * 0.05).bfloat16()
    sl = slice(rank * E // world, (rank + 1) * E // world)
    gx = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(T, h, device=dev, generator=gx).bfloat16()
    ids = torch.randint(0, E, (T, k), device=dev, generator=gx)
    wts = torch.rand(T, k, device=dev, generator=gx)
    outs = []
    for peer in (False, True):
        ep = make_ep_group(dist.group.WORLD, E, device=dev, p2p_bytes=(64 << 20) if peer else 0)
        xi = x.clone().requires_grad_(True)
        wa = w13[sl].clone().requires_grad_(True)
        wb = w2[sl].clone().requires_grad_(True)
        y = moe_forward_ep(xi, wts, ids, wa, wb, ep)
        y.float().square().sum().backward()
        outs.append((y.detach().float(), xi.grad.float(), wa.grad.float(), wb.grad.float()))
    res["moe"] = max(float((p - n).abs().max() / (n.abs().max() + 1e-6)) for p, n in zip(outs[1], outs[0]))
    torch.cuda.synchronize()
    check_errors()
    res["stats"] = dict(a2a.stats)
    q.put(res)
    dist.destroy_process_group()


def test_peer_all_to_all_two_gpus():
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
        assert r["a2a"] == 0.0, r          # a byte copy: exact
        assert r["moe"] < 1e-2, r          # same math, same order: equal up to bf16 reductions
        assert r["stats"]["nccl_fallbacks"] == 0 and r["stats"]["calls"] > 0, r
