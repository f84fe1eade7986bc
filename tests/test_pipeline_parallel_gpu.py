"""Pipeline parallelism on 2 GPUs (NCCL p2p, 1F1B) against the unsplit bf16
decoder on one GPU: every stage's gradients after five micro-batches."""

import os
import socket
from dataclasses import replace

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _loss(lp, ent, mb):
    return -(lp * mb["w"]).sum() / mb["w"].numel()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    from psrl_b200.models import PRESETS, build_model, packed_positions
    from psrl_b200.parallel.pp import PipelineStage
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", rank)
    a = replace(PRESETS["tiny128"], num_layers=4)
    g = torch.Generator().manual_seed(9)
    mbs = []
    for lens in ([300, 129], [512], [64, 64, 200], [1000]):
        T = sum(lens)
        pos, cu, mx = packed_positions(lens, dev)
        mbs.append({"ids": torch.randint(0, a.vocab_size, (T,), generator=g).to(dev), "pos": pos, "cu": cu,
                    "max": mx, "labels": torch.randint(0, a.vocab_size, (T,), generator=g).to(dev),
                    "w": torch.randn(T, generator=g).to(dev)})
    ref = build_model(a, dev, torch.bfloat16, seed=2)
    for mb in mbs:
        lp, ent = ref.logprobs(mb["ids"], mb["pos"], mb["cu"], mb["max"], mb["labels"])
        _loss(lp, ent, mb).backward()
    ref_grads = {n: p.grad.float() for n, p in ref.named_parameters()}
    stage = PipelineStage(build_model(a, dev, torch.bfloat16, seed=2), dist.group.WORLD)
    stage.train_step(mbs, _loss)
    stage.reduce_tied_grads()
    torch.cuda.synchronize()
    worst = max(float((p.grad.float() - ref_grads[n]).abs().max() / (ref_grads[n].abs().max() + 1e-6))
                for n, p in stage.model.named_parameters())
    q.put({"rank": rank, "grad": worst})
    dist.destroy_process_group()


def test_pipeline_two_gpus_matches_one():
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
        assert r["grad"] < 5e-2, r
