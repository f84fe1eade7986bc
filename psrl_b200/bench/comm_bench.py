"""Collective and link micro-benchmarks (C38: the reference's cluster scanner
runs an NCCL all-reduce microbenchmark and discovers links,
``psrl/bench/basic/`` ``MicrobenchRunner``).

Run one process per GPU::

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m psrl_b200.bench.comm_bench --sizes-mb 1,16,256,1024

Reports, per message size, the device time (CUDA events on the launching
stream, max over ranks) and the bus bandwidth of

* ``all_reduce``      (busbw = bytes * 2 (n-1)/n / t),
* ``all_gather``      (busbw = bytes * (n-1)/n / t, bytes = gathered size),
* ``reduce_scatter``  (busbw = bytes * (n-1)/n / t, bytes = input size),
* ``peer_pull``       rank r pulls ``bytes`` from rank (r+1) % n with the
  repository's peer-load kernel (CUDA IPC mapping, 16-byte loads over NVLink),

plus the link inventory (``nvidia-smi topo -m`` and NVML NVLink state, read
only).  Inputs are larger than L2 from 256 MB on; smaller sizes measure
latency.  One JSON object per line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess

import torch
import torch.distributed as dist


def link_inventory() -> dict:
    out: dict = {}
    try:
        out["topo"] = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True,
                                     timeout=30).stdout
    except (OSError, subprocess.SubprocessError) as exc:
        out["topo_error"] = str(exc)
    try:
        import pynvml
        pynvml.nvmlInit()
        links = []
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            up = 0
            for link in range(18):
                try:
                    if pynvml.nvmlDeviceGetNvLinkState(h, link) == pynvml.NVML_FEATURE_ENABLED:
                        up += 1
                except pynvml.NVMLError:
                    break
            links.append({"gpu": i, "nvlinks_up": up})
        out["nvlink"] = links
        pynvml.nvmlShutdown()
    except Exception as exc:        # NVML is optional (CPU boxes, containers)
        out["nvml_error"] = str(exc)
    return out


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier(device_ids=[torch.cuda.current_device()])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="1,16,256,1024")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--ops", default="all_reduce,all_gather,reduce_scatter,peer_pull")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, n = dist.get_rank(), dist.get_world_size()
    ops = args.ops.split(",")
    if rank == 0:
        print(json.dumps({"links": link_inventory(), "world": n}), flush=True)
    for mb in [float(x) for x in args.sizes_mb.split(",")]:
        nbytes = int(mb * 2**20) // (16 * n) * (16 * n)
        numel = nbytes // 2
        x = torch.randn(numel, device="cuda").bfloat16()
        res = {"bytes": nbytes, "world": n}
        if "all_reduce" in ops:
            ms = _time(lambda: dist.all_reduce(x), args.iters, args.warmup)
            res["all_reduce"] = {"ms": ms, "busbw_gbs": nbytes * 2 * (n - 1) / n / (ms / 1e3) / 1e9}
        if "all_gather" in ops:
            shard = x[: numel // n]
            outp = torch.empty_like(x)
            ms = _time(lambda: dist.all_gather_into_tensor(outp, shard), args.iters, args.warmup)
            res["all_gather"] = {"ms": ms, "busbw_gbs": nbytes * (n - 1) / n / (ms / 1e3) / 1e9}
        if "reduce_scatter" in ops:
            outs = torch.empty(numel // n, device="cuda", dtype=x.dtype)
            ms = _time(lambda: dist.reduce_scatter_tensor(outs, x), args.iters, args.warmup)
            res["reduce_scatter"] = {"ms": ms, "busbw_gbs": nbytes * (n - 1) / n / (ms / 1e3) / 1e9}
        if "peer_pull" in ops and n > 1:
            from ..parallel.weight_sync import WeightLayout, WeightPuller, WeightStore
            layout = WeightLayout([("w", (numel,), 0)], numel, torch.bfloat16)
            store = WeightStore(layout, torch.device("cuda", local), "hbm")
            store.publish(x, 0)
            torch.cuda.synchronize()
            descs: list = [None] * n
            dist.all_gather_object(descs, store.descriptor())
            dst = torch.empty_like(x)
            puller = WeightPuller(layout, [descs[(rank + 1) % n]], dst)
            ms = _time(puller.pull, args.iters, args.warmup)
            res["peer_pull"] = {"ms": ms, "gbs": nbytes / (ms / 1e3) / 1e9}
            del puller
            dist.barrier(device_ids=[local])
        if rank == 0:
            print(json.dumps(res), flush=True)
        del x
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
