"""Fused data-parallel optimizer step over NVLink peer memory (K13/K14).

:class:`PeerShardedStep` replaces FlatShardedDP's NCCL reduce-scatter, AdamW
and all-gather with two kernels (``csrc/peer_optim.cu``):

1. ``peer_reduce``  — this rank's shard of every bucket is summed straight out
   of every rank's fp32 gradient buffer (CUDA IPC mappings, 16-byte peer
   loads), producing the reduced shard and its squared norm in one pass;
2. NCCL all-reduce of the squared norm (one float) and the clip coefficient;
3. ``peer_adamw``   — AdamW on the fp32 master shard with the clipped reduced
   gradient, and the bf16 result stored into EVERY rank's parameter buffer
   (the all-gather fused into the update's store).

Ordering between ranks comes from one-element NCCL all-reduces on the same
stream before step 1 (every rank finished its backward) and after step 3
(every rank's peer stores landed before anyone's next forward); the norm
all-reduce separates 1 and 3 (every rank finished reading the gradients).  No
kernel spins on another rank, and there is no TMA or multicast anywhere.

Traffic equals the NCCL path (each rank reads its shard from N-1 peers and
writes its bf16 shard to N-1 peers), minus the separate passes over the
reduced shard that reduce-scatter, AdamW and all-gather make one after another.
Reference: the FSDP2 reduce-scatter + optimizer step of the engine train worker
(``psrl/workers/train/engine_train_worker.py``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops


class PeerShardedStep:
    def __init__(self, dp):
        self.dp = dp
        g = dp.group
        ext = ops.ext()
        world, rank = dp.world, dp.rank
        # exchange IPC handles of the gradient and parameter buffers
        mine = {"grad": ext.ipc_handle(dp.flat_grad), "flat": ext.ipc_handle(dp.flat),
                "device": dp.device.index, "total": dp.total}
        allh: list = [None] * world
        dist.all_gather_object(allh, mine, group=g)
        self.grads, self.flats = [], []
        for r, h in enumerate(allh):
            if int(h["total"]) != dp.total:
                raise RuntimeError("peer optimizer: flat buffers differ across ranks")
            if r == rank:
                self.grads.append(dp.flat_grad)
                self.flats.append(dp.flat)
            else:
                gh, goff = h["grad"]
                fh, foff = h["flat"]
                self.grads.append(ext.ipc_open(gh, int(goff), dp.total, torch.float32, int(h["device"])))
                self.flats.append(ext.ipc_open(fh, int(foff), dp.total, dp.flat.dtype, int(h["device"])))
        starts, srcs = [0], []
        for b in dp.buckets:
            srcs.append(b.base + b.lo)
            starts.append(starts[-1] + b.shard)
        if starts[-1] != dp.shard_total:
            raise RuntimeError("peer optimizer: shard layout mismatch")
        dev = dp.device
        self.start = torch.tensor(starts, dtype=torch.int64, device=dev)
        self.src_off = torch.tensor(srcs, dtype=torch.int64, device=dev)
        self.sq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.partial = torch.empty(1024, dtype=torch.float32, device=dev)
        self.tick = torch.zeros(1, dtype=torch.float32, device=dev)

    def _fence(self) -> None:
        # stream-ordered rendezvous: completes on a rank only once every rank
        # reached it, i.e. after all of their earlier work on this stream
        dist.all_reduce(self.tick, group=self.dp.group)

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0) -> dict:
        dp = self.dp
        ext = ops.ext()
        self._fence()
        ext.peer_reduce(self.grads, self.flats, self.start, self.src_off, dp.grad_shard_all, self.sq, self.partial)
        dist.all_reduce(self.sq, group=dp.group)
        if grad_scale != 1.0:
            self.sq.mul_(grad_scale * grad_scale)
        dp.norm.sq.copy_(self.sq)
        coef, gnorm = dp.norm.clip_coef(dp.max_grad_norm)
        lr = dp.current_lr()
        b1, b2 = dp.betas
        ext.peer_adamw(self.grads, self.flats, self.start, self.src_off, dp.master_all, dp.grad_shard_all, dp.m_all,
                       dp.v_all, lr, b1, b2, dp.eps, dp.wd, dp.step_count, coef, grad_scale)
        self._fence()
        dp.zero_grad()
        return {"grad_norm": gnorm, "lr": lr}
