"""Sharded data parallelism with flat buckets (the trainer's FSDP backend).

Layout (chosen for 180 GB of HBM per GPU):

* every rank keeps the **full bf16 parameters** resident (views into one flat
  buffer per bucket, one bucket per decoder layer), so forward/backward never
  wait for a parameter all-gather;
* gradients are accumulated across micro-batches into **fp32 main-grad**
  buckets (post-accumulate hooks turn each bf16 ``.grad`` into an fp32 add);
* the fp32 **master weights and Adam moments are sharded** 1/world per bucket
  (ZeRO-2 style optimizer-state sharding);
* the optimizer step per bucket is: reduce-scatter(grad) → global grad-norm
  (one tiny all-reduce) → fused AdamW on the shard writing the bf16 shard in
  place → all-gather of the bf16 shard back into the full bucket.

``shard_grads=True`` (gradient sharding, for models whose full fp32 main
gradients would not fit beside the rest): there is no model-wide gradient
buffer.  A bucket's gradients accumulate into a transient fp32 staging buffer
of one bucket; when the backward has produced all of them the staging buffer
is reduce-scattered and added into this rank's fp32 gradient shard, and
freed.  One reduce-scatter per bucket per micro-batch (issued from the
backward, in bucket-completion order, which is the same on every rank of a
dense model) instead of one per step; the peer-memory step, which reads every
peer's full gradient buffer, is off in this mode.

The reference trains with FSDP2 full-shard (parameters re-gathered per layer
in every forward and backward, ``engine_train_worker.py:80-85``); keeping
parameters resident trades 2 bytes/param of HBM for one all-gather per
optimizer step instead of two per micro-batch.  Collectives here are NCCL
(the baseline path); :mod:`psrl_b200.parallel.peer` provides the fused
peer-memory path (one kernel reduces this rank's shard from every peer's
gradient buffer over NVLink, one kernel runs AdamW on it and stores the bf16
shard into every peer's parameter buffer).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import ops


class _Bucket:
    def __init__(self, names, params, world: int, rank: int, device, pad_to: int, flat: torch.Tensor,
                 grad: torch.Tensor, base: int, shard_bufs: tuple, shard_start: int):
        self.names = names
        self.params = params
        n = sum(p.numel() for p in params)
        self.numel = n
        padded = math.ceil(n / pad_to) * pad_to
        self.padded = padded
        self.shard = padded // world
        self.rank = rank
        self.base = base                     # offset of this bucket in the model-wide flat buffer
        self.flat = flat[base: base + padded]
        self.grad = grad[base: base + padded] if grad.numel() else None
        self.stage = None                    # gradient sharding: this bucket's fp32 staging buffer
        self.fired: set = set()
        off = 0
        self.offsets = []
        for p in params:
            k = p.numel()
            self.flat[off: off + k].copy_(p.data.reshape(-1))
            p.data = self.flat[off: off + k].view(p.shape)
            self.offsets.append(off)
            off += k
        lo = rank * self.shard
        self.lo, self.hi = lo, lo + self.shard
        # this rank's shard of the bucket: views into model-wide contiguous shard
        # buffers (master, m, v, reduced grad), so one kernel can sweep them all
        master_all, m_all, v_all, gs_all = shard_bufs
        self.shard_start = shard_start
        sl = slice(shard_start, shard_start + self.shard)
        self.master = master_all[sl]
        self.master.copy_(self.flat[lo: self.hi].float())
        self.m = m_all[sl]
        self.v = v_all[sl]
        self.grad_shard = self.grad[lo: self.hi] if world == 1 else gs_all[sl]
        self.params_set = set(id(p) for p in params)

    def param_shard(self) -> torch.Tensor:
        return self.flat[self.lo: self.hi]


class FlatShardedDP:
    def __init__(self, model: torch.nn.Module, group=None, *, lr: float = 1e-6, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_grad_norm: float = 1.0, warmup_steps: int = 0,
                 bucket_mode: str = "layer", param_filter=None, norm_group=None, count_in_norm: bool = True,
                 replicate_group=None, shard_grads: bool = False):
        """``param_filter(name) -> bool`` selects the parameters this instance
        owns (default: all trainable ones).  ``norm_group``: ranks whose
        parameters are disjoint from this rank's (expert parallelism), summed
        into the squared gradient norm in addition to ``group``'s shards.
        ``count_in_norm=False``: the parameters are a copy of ones another rank
        already counts (a tied embedding on the last pipeline stage): they are
        reduced and updated but add nothing to the clip norm.
        ``replicate_group`` (hybrid sharding, HSDP): ``group`` is this rank's
        shard group and ``replicate_group`` the ranks holding the same shard in
        the other shard groups; the reduce-scattered shard is summed over it
        before the update, so every replica applies the same step."""
        self.model = model
        self.group = group
        self.replicate_group = replicate_group if (replicate_group is not None and dist.is_initialized()
                                                   and dist.get_world_size(replicate_group) > 1) else None
        self.norm_group = norm_group
        self.count_in_norm = bool(count_in_norm)
        # no group = this rank trains alone (even inside a larger job)
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.shard_grads = bool(shard_grads) and self.world > 1
        self.device = next(model.parameters()).device
        self.lr, self.betas, self.eps, self.wd = lr, tuple(betas), eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.warmup_steps = warmup_steps
        self.step_count = 0
        pad_to = self.world * 64
        groups: dict[str, list] = {}
        order: list[str] = []
        for name, p in model.named_parameters():
            if not p.requires_grad or (param_filter is not None and not param_filter(name)):
                continue
            key = ".".join(name.split(".")[:2]) if (bucket_mode == "layer" and name.startswith("layers.")) else "misc"
            if key not in groups:
                groups[key] = []
                order.append(key)
            groups[key].append((name, p))
        self.buckets: list[_Bucket] = []
        self.param_to_bucket: dict = {}
        # one model-wide flat buffer (parameters) and one fp32 flat buffer (main grads);
        # buckets are padded slices so every shard boundary is 64-element aligned
        sizes = [math.ceil(sum(p.numel() for _, p in groups[k]) / pad_to) * pad_to for k in order]
        self.total = sum(sizes)
        dtype = next(model.parameters()).dtype
        self.num_params = sum(p.numel() for k in order for _, p in groups[k])
        self.flat = torch.zeros(self.total, dtype=dtype, device=self.device)
        # the model-wide fp32 main-grad buffer (a placeholder when gradients are sharded)
        self.flat_grad = torch.zeros(self.total if not self.shard_grads else 0, dtype=torch.float32,
                                     device=self.device)
        self.shard_total = self.total // self.world
        f32 = dict(dtype=torch.float32, device=self.device)
        self.master_all = torch.zeros(self.shard_total, **f32)
        self.m_all = torch.zeros(self.shard_total, **f32)
        self.v_all = torch.zeros(self.shard_total, **f32)
        self.grad_shard_all = torch.zeros(self.shard_total if self.world > 1 else 0, **f32)
        bufs = (self.master_all, self.m_all, self.v_all, self.grad_shard_all)
        base = 0
        shard_start = 0
        self.layout: list[tuple[str, tuple, int]] = []   # (name, shape, offset) in the flat buffer
        for key, sz in zip(order, sizes):
            names = [n for n, _ in groups[key]]
            params = [p for _, p in groups[key]]
            b = _Bucket(names, params, self.world, self.rank, self.device, pad_to, self.flat, self.flat_grad, base,
                        bufs, shard_start)
            for nm, p, off in zip(names, params, b.offsets):
                self.layout.append((nm, tuple(p.shape), base + off))
            base += sz
            shard_start += b.shard
            for i, p in enumerate(params):
                self.param_to_bucket[p] = (b, b.offsets[i])
            self.buckets.append(b)
        self._hooks = [p.register_post_accumulate_grad_hook(self._accumulate) for p in self.param_to_bucket]
        self.norm = ops.NormAccumulator(self.device)
        self.peer = None            # peer-memory step (parallel.peer.PeerShardedStep), set by enable_peer_step

    def enable_peer_step(self) -> bool:
        """Use the fused peer-memory reduce-scatter + AdamW + all-gather kernels
        for the optimizer step (CUDA, world > 1).  Returns whether it is on."""
        if self.world <= 1 or self.device.type != "cuda" or self.replicate_group is not None or self.shard_grads:
            return False
        from .peer import PeerShardedStep
        self.peer = PeerShardedStep(self)
        return True

    # --------------------------------------------------------------- grads
    def _accumulate(self, p: torch.Tensor) -> None:
        b, off = self.param_to_bucket[p]
        if not self.shard_grads:
            b.grad[off: off + p.numel()].add_(p.grad.reshape(-1))
            p.grad = None
            return
        if b.stage is None:
            b.stage = torch.zeros(b.padded, dtype=torch.float32, device=self.device)
        b.stage[off: off + p.numel()].add_(p.grad.reshape(-1))
        p.grad = None
        b.fired.add(id(p))
        if len(b.fired) == len(b.params_set):
            self._flush(b)

    def _flush(self, b) -> None:
        """Gradient sharding: reduce-scatter a bucket's staged gradients into
        this rank's shard and free the staging buffer."""
        part = torch.empty(b.shard, dtype=torch.float32, device=self.device)
        dist.reduce_scatter_tensor(part, b.stage, op=dist.ReduceOp.SUM, group=self.group)
        b.grad_shard.add_(part)
        b.stage = None
        b.fired = set()

    def zero_grad(self) -> None:
        if self.shard_grads:
            self.grad_shard_all.zero_()
            for b in self.buckets:
                b.stage, b.fired = None, set()
        else:
            self.flat_grad.zero_()

    # ---------------------------------------------------------------- step
    def current_lr(self) -> float:
        if self.warmup_steps > 0:
            return self.lr * min(1.0, (self.step_count + 1) / self.warmup_steps)
        return self.lr

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, partners: list | None = None) -> dict:
        """Reduce, clip, update, re-gather.  Gradients are *summed* across ranks
        (callers normalise the loss by the global token/sequence count).
        ``partners``: other FlatShardedDP instances of the same model (e.g. the
        expert-parallel parameters) stepped with one shared clip coefficient."""
        group_all = [self] + list(partners or [])
        for d in group_all:
            d.step_count += 1
        if self.peer is not None and not partners:
            return self.peer.step(grad_scale)
        sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        for d in group_all:
            sq += d.reduce_grads()
        if grad_scale != 1.0:
            sq.mul_(grad_scale * grad_scale)
        self.norm.sq.copy_(sq)
        coef, gnorm = self.norm.clip_coef(self.max_grad_norm)
        lr = self.current_lr()
        for d in group_all:
            d.apply_update(coef, lr, grad_scale)
        return {"grad_norm": gnorm, "lr": lr}

    @torch.no_grad()
    def reduce_grads(self) -> torch.Tensor:
        """Reduce-scatter the main grads into this rank's shards; returns the
        global squared norm of this instance's gradients (device scalar)."""
        self.norm.reset()
        if self.shard_grads:
            # buckets some of whose parameters got no gradient: flush in bucket
            # order (the same set on every rank of a dense model)
            for b in self.buckets:
                if b.stage is not None:
                    self._flush(b)
        for b in self.buckets:
            if self.world > 1 and not self.shard_grads:
                dist.reduce_scatter_tensor(b.grad_shard, b.grad, op=dist.ReduceOp.SUM, group=self.group)
            if self.replicate_group is not None:
                dist.all_reduce(b.grad_shard, group=self.replicate_group)
            self.norm.add(b.grad_shard)
        if self.world > 1:
            dist.all_reduce(self.norm.sq, group=self.group)
        if self.norm_group is not None:
            dist.all_reduce(self.norm.sq, group=self.norm_group)
        if not self.count_in_norm:
            return torch.zeros_like(self.norm.sq)
        return self.norm.sq.clone()

    @torch.no_grad()
    def apply_update(self, coef: torch.Tensor, lr: float, grad_scale: float = 1.0) -> None:
        b1, b2 = self.betas
        for b in self.buckets:
            ops.adamw_(b.master, b.grad_shard, b.m, b.v, b.param_shard(), lr, b1, b2, self.eps, self.wd,
                       self.step_count, coef, grad_scale)
            if self.world > 1:
                dist.all_gather_into_tensor(b.flat, b.param_shard(), group=self.group)
        self.zero_grad()

    # -------------------------------------------------------------- state
    def full_params(self) -> dict[str, torch.Tensor]:
        return dict(self.model.named_parameters())

    def optimizer_state(self) -> dict:
        return {
            "step": self.step_count,
            "buckets": [{"names": b.names, "master": b.master.cpu(), "m": b.m.cpu(), "v": b.v.cpu()}
                        for b in self.buckets],
            "world": self.world,
            "rank": self.rank,
        }

    def load_optimizer_state(self, st: dict) -> None:
        if st.get("world") != self.world:
            raise ValueError("optimizer state was saved with a different world size")
        self.step_count = int(st["step"])
        for b, s in zip(self.buckets, st["buckets"]):
            if s["names"] != b.names:
                raise ValueError("optimizer state bucket mismatch")
            b.master.copy_(s["master"])
            b.m.copy_(s["m"])
            b.v.copy_(s["v"])

    @torch.no_grad()
    def sync_master_from_params(self) -> None:
        """After loading bf16 params from a checkpoint, refresh the fp32 master shards."""
        for b in self.buckets:
            b.master.copy_(b.param_shard().float())

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()


def hybrid_shard_groups(group, shard_size: int):
    """(shard group, replicate group) of this rank for hybrid sharding over
    ``group``: shard groups of ``shard_size`` consecutive ranks of ``group``,
    replicate groups of the ranks at the same position in each.  Only the
    ranks of ``group`` take part (local synchronisation), so a trainer group
    inside a larger job can call it alone."""
    world = dist.get_world_size(group)
    if shard_size <= 0 or shard_size >= world:
        return group, None
    if world % shard_size:
        raise ValueError(f"{world} data-parallel ranks do not split into shard groups of {shard_size}")
    ranks = dist.get_process_group_ranks(group)
    me = dist.get_rank(group)
    shard = rep = None
    for i in range(world // shard_size):
        g = dist.new_group(ranks[i * shard_size:(i + 1) * shard_size], use_local_synchronization=True) \
            if me // shard_size == i else None
        shard = g if g is not None else shard
    for j in range(shard_size):
        if me % shard_size == j:
            rep = dist.new_group(ranks[j::shard_size], use_local_synchronization=True)
    return shard, rep
