"""Process-group plumbing: one process per GPU, NCCL on GPU and gloo on CPU.

Role layout for the asynchronous RL job on one node: ranks ``[0, n_train)``
train, ranks ``[n_train, world)`` serve rollout; with a single process both
roles share the device (colocated).  Rendezvous always uses 127.0.0.1.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    device: torch.device = torch.device("cpu")
    backend: str = "gloo"

    @property
    def is_dist(self) -> bool:
        return self.world_size > 1


def init_distributed(device: str = "auto", timeout_s: float = 600.0) -> DistInfo:
    """Initialise the default process group from torchrun env vars (if present)."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    use_cuda = torch.cuda.is_available() if device == "auto" else device.startswith("cuda")
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        backend = "nccl"
    else:
        dev = torch.device("cpu")
        backend = "gloo"
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        # lazy NCCL communicator creation (no device_id binding): subgroups are then
        # created only by their members, without a collective over the world
        dist.init_process_group(backend=backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
    return DistInfo(rank, world, local, dev, backend)


def new_subgroup(ranks: list[int], backend: str | None = None):
    """Create a subgroup; only member ranks call this (group-local synchronisation)."""
    if not dist.is_initialized():
        return None
    return dist.new_group(ranks=ranks, backend=backend, use_local_synchronization=True)


def broadcast_value(v, src: int = 0, group=None):
    """Broadcast a picklable value from ``src`` (identity without a process group)."""
    if not dist.is_initialized():
        return v
    box = [v]
    dist.broadcast_object_list(box, src=src, group=group)
    return box[0]


def barrier(group=None):
    if dist.is_initialized():
        if dist.get_backend(group) == "nccl" and torch.cuda.is_available():
            dist.barrier(group=group, device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier(group=group)


def all_reduce_max(x: float, device, group=None) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def all_reduce_sum(x: float, device, group=None) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item())


def destroy():
    if dist.is_initialized():
        dist.destroy_process_group()
