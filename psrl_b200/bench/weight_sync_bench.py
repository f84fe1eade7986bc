"""Trainer -> rollout weight-sync sweep (K17 / the agentic config's sync
sweep): one trainer rank publishes a bf16 parameter store of ``--gb`` GB in
its HBM; every other rank is a rollout replica that pulls the whole store
over NVLink with the repository's peer-load kernel (CUDA IPC mapping,
16-byte loads, no staging, no multicast).  Replicas pull concurrently, as after
a version bump.

Run one process per GPU::

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m psrl_b200.bench.weight_sync_bench --gb 15.2

Reported per replica count: the device time of one sync (CUDA events on each
replica, max over replicas, after warm-up), the bandwidth each replica gets,
and the fraction of the NVLink roofline.  The roofline time is the larger of
two bounds:

- the source GPU sending ``gb x replicas`` bytes at 770 GB/s (the measured
  per-direction peer copy bandwidth);
- one replica receiving ``gb`` bytes at 770 GB/s.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0   # measured peer copy per direction per GPU on this hardware


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gb", type=float, default=15.2)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from ..parallel.weight_sync import WeightLayout, WeightPuller, WeightStore
    numel = int(args.gb * 1e9 / 2) // 64 * 64
    layout = WeightLayout([("w", (numel,), 0)], numel, torch.bfloat16)
    desc = None
    if rank == 0:
        src = torch.randn(numel // 64, device="cuda").bfloat16().repeat_interleave(64)
        store = WeightStore(layout, torch.device("cuda", local), "hbm")
        store.publish(src, 1)
        del src
        torch.cuda.synchronize()
        desc = store.descriptor()
    box = [desc]
    dist.broadcast_object_list(box, src=0)
    results = []
    for replicas in range(1, world):
        puller = None
        if 1 <= rank <= replicas:
            dst = torch.empty(numel, device="cuda", dtype=torch.bfloat16)
            puller = WeightPuller(layout, [box[0]], dst)
            for _ in range(args.warmup):
                puller.pull()
            torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        ms = 0.0
        if puller is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iters):
                puller.pull()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.iters
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        nbytes = numel * 2
        roof_s = max(nbytes * replicas / (LINK_GBS * 1e9), nbytes / (LINK_GBS * 1e9))
        res = {"replicas": replicas, "gb": round(nbytes / 1e9, 2), "ms": round(ms, 2),
               "per_replica_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
               "roofline_ms": round(roof_s * 1e3, 2), "frac_roofline": round(roof_s * 1e3 / ms, 3)}
        results.append(res)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if puller is not None:
            del puller, dst
            torch.cuda.empty_cache()
        dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
