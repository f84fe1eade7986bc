"""Step strategies: how one training step pipelines its stages (C3).

``STAGE_META`` tags each stage:

* ``per_sample``     — may run on a chunk as soon as it arrives (old/ref
  log-probs, values, reward);
* ``batch_coupled``  — needs the whole (group-complete) batch (advantages);
* ``optimizer_step`` — parameter updates.

``FullBatchStepStrategy`` waits for the whole staleness buffer, then runs the
stages in order.  ``FineGrainOverlapStrategy`` consumes the buffer in chunks
while it fills: with ``overlap_scope=recompute`` the per-sample stages run on
each arrived chunk (their cost hides under rollout time); with
``overlap_scope=pre_step`` at ``mini_batch`` granularity each arrived
mini-batch is also advantage-normalised and trained on immediately (its own
optimizer step).  Reference: ``psrl/trainer/ppo/strategies/``.
"""

from __future__ import annotations

import time

from . import algos

STAGE_META: dict[str, str] = {
    "old_log_prob": "per_sample",
    "ref_log_prob": "per_sample",
    "values": "per_sample",
    "reward": "per_sample",
    "advantage": "batch_coupled",
    "update_actor": "optimizer_step",
    "update_critic": "optimizer_step",
}


class StepStrategy:
    def __init__(self, trainer):
        self.t = trainer

    # per-sample stages on a list of trajectories
    def per_sample(self, trajs) -> None:
        t = self.t
        idx = list(range(len(trajs)))
        if not trajs:
            return
        if t.critic is not None:
            t.critic.compute_values(trajs, idx)
        if t.ref is not None:
            t.ref.compute_log_prob(trajs, idx, field="ref_logprobs")
        if not t.cfg.psrl.log_prob.enable_rollout_engine_log_prob:
            t.actor.compute_log_prob(trajs, idx, field="old_logprobs")
        else:
            for x in trajs:
                x.old_logprobs = x.rollout_logprobs

    def optimize(self, trajs, metrics: dict) -> None:
        from .driver import compute_batch_advantages
        t = self.t
        metrics.update(compute_batch_advantages(t.cfg, trajs, getattr(t, "kl_ctrl", None)))
        metrics.update(algos.apply_rollout_correction(t.cfg.algorithm.rollout_correction, trajs))
        with t.log.span("TRAIN", step=t.global_step):
            if t.critic is not None:
                metrics.update(t.critic.update_critic(trajs))
            metrics.update(t.actor.update_policy(
                trajs, float(t.cfg.rollout.temperature),
                step_guard=t._push_guard() if t.overlap else None, sync_every_micro_batch=t.overlap))

    def run_step(self, buffer_id: int, metrics: dict):
        raise NotImplementedError


class FullBatchStepStrategy(StepStrategy):
    def run_step(self, buffer_id, metrics):
        t0 = time.perf_counter()
        with self.t.log.span("GEN", step=buffer_id):
            self.t.wait_for_buffer(buffer_id)
        t1 = time.perf_counter()
        trajs = self.t.manager.consume(buffer_id)
        self.per_sample(trajs)
        self.optimize(trajs, metrics)
        metrics["timing_s/gen_wait"] = t1 - t0
        metrics["timing_s/train"] = time.perf_counter() - t1
        return trajs


def resolve_fine_grain_chunk_size(cfg) -> tuple[str, int]:
    fgo = cfg.psrl.fine_grain_overlap
    mini = int(cfg.actor.ppo_mini_batch_size)
    if fgo.granularity == "mini_batch":
        return "mini_batch", max(1, mini)
    mult = max(1, int(fgo.multiplier))
    return "micro_batch", max(1, mini // mult)


class FineGrainOverlapStrategy(StepStrategy):
    def __init__(self, trainer):
        super().__init__(trainer)
        self.granularity, self.chunk_groups = resolve_fine_grain_chunk_size(trainer.cfg)
        self.scope = trainer.cfg.psrl.fine_grain_overlap.overlap_scope
        if self.scope == "pre_step" and self.granularity != "mini_batch":
            raise ValueError("pre_step overlap needs mini_batch granularity")

    def run_step(self, buffer_id, metrics):
        t = self.t
        t0 = time.perf_counter()
        done_entries = 0
        trained: list = []
        nchunks = 0
        ready_entries = t.manager.ready_entries
        if t.overlap:
            t.start_rollout()
        while True:
            ready = t.manager.buffer_ready(buffer_id)
            avail = t.manager.occupied_prefix(buffer_id)
            while avail - done_entries >= self.chunk_groups or (ready and avail > done_entries):
                n = min(self.chunk_groups, avail - done_entries)
                chunk = t.manager.peek(buffer_id, done_entries, done_entries + n)
                self.per_sample(chunk)
                if self.scope == "pre_step":
                    self.optimize(chunk, metrics)
                    trained.extend(chunk)
                nchunks += 1
                done_entries += n
            if ready and done_entries >= ready_entries:
                break
            if not t.overlap:
                t.instance.pump()
            else:
                time.sleep(0.002)
        t1 = time.perf_counter()
        trajs = t.manager.consume(buffer_id)
        if self.scope != "pre_step":
            self.optimize(trajs, metrics)
        metrics["timing_s/gen_wait"] = t1 - t0
        metrics["timing_s/train"] = time.perf_counter() - t1
        metrics["fine_grain/chunks"] = nchunks
        return trajs


def build_step_strategy(trainer) -> StepStrategy:
    if trainer.cfg.psrl.fine_grain_overlap.granularity == "none":
        return FullBatchStepStrategy(trainer)
    return FineGrainOverlapStrategy(trainer)


# --------------------------------------------- multi-GPU placements (sharded)


def per_sample_missing(cfg, trajs, actor, ref=None, critic=None) -> None:
    """Per-sample stages on trajectories that do not carry their result yet
    (reference log-probs, old log-probs unless the rollout engine's are used,
    critic values).  Every worker call runs even with nothing to do, so
    expert- and tensor-parallel forwards stay matched across ranks."""
    if ref is not None:
        ref.compute_log_prob(trajs, [i for i, t in enumerate(trajs) if t.ref_logprobs is None], field="ref_logprobs")
    if not bool(cfg.psrl.log_prob.enable_rollout_engine_log_prob):
        actor.compute_log_prob(trajs, [i for i, t in enumerate(trajs) if t.old_logprobs is None],
                               field="old_logprobs")
    if critic is not None:
        critic.compute_values(trajs, [i for i, t in enumerate(trajs) if t.old_values is None])


def sharded_overlap_mode(cfg) -> str | None:
    """None, ``"recompute"`` or ``"pre_step"`` for the multi-GPU placements.
    ``pre_step`` trains each mini-batch as soon as it is committed, so it
    needs ``mini_batch`` granularity and batch-free advantages: no critic
    and no in-reward KL (both need the whole batch's statistics)."""
    fgo = cfg.psrl.fine_grain_overlap
    if fgo.granularity == "none":
        return None
    if fgo.overlap_scope == "pre_step":
        if fgo.granularity != "mini_batch":
            raise ValueError("pre_step overlap needs psrl.fine_grain_overlap.granularity=mini_batch")
        if cfg.critic.enable or cfg.algorithm.get("use_kl_in_reward"):
            raise ValueError("pre_step overlap in the multi-GPU placements takes outcome estimators without "
                             "a critic or in-reward KL")
        return "pre_step"
    return "recompute"


def pre_step_train(cfg, cp, b: int, actor, ref=None, *, group=None, src: int = 0, dp_rank: int = 0,
                   dp_world: int = 1, step_guard=None, sync_every_micro_batch: bool = False,
                   poll_s: float = 0.01, timeout_s: float = 1800.0) -> tuple[dict, int]:
    """``overlap_scope=pre_step`` in the multi-GPU placements: each committed
    mini-batch of buffer ``b`` is trained (one optimizer step) as soon as it
    arrives, while the rest of the buffer is still being generated.

    Every trainer rank takes the same chunk (rank ``src`` broadcasts the
    buffer's progress over ``group``) and computes its advantages over the
    whole chunk (the chunk holds complete prompt groups); the chunk is split
    into token-balanced data-parallel shares as a full batch would be, and
    each rank computes the per-sample stages and the update on its share.
    The caller consumes the buffer afterwards (its batch is not trained
    again).  Returns (averaged actor metrics, chunks)."""
    import torch.distributed as dist

    from .actor import plan_update
    from .driver import compute_batch_advantages
    _, chunk = resolve_fine_grain_chunk_size(cfg)
    use_rl = bool(cfg.psrl.log_prob.enable_rollout_engine_log_prob)
    sums: dict = {}
    t0 = time.monotonic()
    done = chunks = 0
    while True:
        lead = group is None or dist.get_rank() == src
        msg = [cp.progress(b) if lead else None]
        if group is not None:
            dist.broadcast_object_list(msg, src=src, group=group)
        avail, ready, _need = msg[0]
        if avail - done >= chunk or (ready and avail > done):
            hi = min(int(avail), done + chunk)
            trajs = cp.peek_chunk(b, done, hi)
            for t in trajs:
                t.old_logprobs = t.rollout_logprobs if use_rl else None
            adv_m = compute_batch_advantages(cfg, trajs)
            plans = plan_update(trajs, len(trajs) + 1, dp_world)
            need = sorted({i for mine, _, _ in plans[dp_rank] for i in mine})
            local = {g: j for j, g in enumerate(need)}
            mine = [trajs[i] for i in need]
            plan = [([local[i] for i in idx], gt, ns) for idx, gt, ns in plans[dp_rank]]
            per_sample_missing(cfg, mine, actor, ref, None)
            m = dict(adv_m)
            m.update(algos.apply_rollout_correction(cfg.algorithm.rollout_correction, mine))
            m.update(actor.update_policy(mine, float(cfg.rollout.temperature), step_guard=step_guard,
                                         sync_every_micro_batch=sync_every_micro_batch, plan=plan))
            for k, v in m.items():
                sums.setdefault(k, []).append(float(v))
            done = hi
            chunks += 1
            t0 = time.monotonic()
        elif ready:
            if group is not None:
                dist.barrier(group=group)
            return {k: sum(v) / len(v) for k, v in sums.items()}, chunks
        else:
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"buffer {b}: no progress for the pre_step overlap")
            time.sleep(poll_s)


def sharded_overlap_enabled(cfg) -> bool:
    return sharded_overlap_mode(cfg) == "recompute"


def overlap_per_sample(cfg, cp, b: int, compute, *, group=None, src: int = 0, dp_rank: int = 0, dp_world: int = 1,
                       post: bool = True, poll_s: float = 0.01, timeout_s: float = 1800.0) -> int:
    """Fine-grain overlap (``overlap_scope=recompute``) in the multi-GPU
    placements: while staleness buffer ``b`` fills, the trainer ranks run the
    per-sample stages on each committed chunk of entries and post the results
    to the control plane, which attaches them when it builds the batch; the
    step then computes only what is still missing.

    Rank ``src`` polls the buffer's progress and broadcasts it over ``group``
    (trainer ranks, gloo), so every rank takes the same chunks.  Each data-
    parallel rank takes every ``dp_world``-th trajectory of a chunk (the
    tensor-parallel ranks of one data-parallel rank compute it together;
    ``post`` is set on one of them).  Returns the number of chunks.
    Reference: ``psrl/trainer/ppo/strategies/`` (fine-grain overlap)."""
    import torch.distributed as dist
    _, chunk = resolve_fine_grain_chunk_size(cfg)
    t0 = time.monotonic()
    done = chunks = 0
    while True:
        lead = group is None or dist.get_rank() == src
        msg = [cp.progress(b) if lead else None]
        if group is not None:
            dist.broadcast_object_list(msg, src=src, group=group)
        avail, ready, _need = msg[0]
        if avail - done >= chunk or (ready and avail > done):
            hi = min(int(avail), done + chunk)
            trajs = cp.peek_chunk(b, done, hi)
            mine = [t for i, t in enumerate(trajs) if i % dp_world == dp_rank]
            compute(mine)
            if post:
                fields = {}
                for t in mine:
                    f = {k: getattr(t, k) for k in ("old_logprobs", "ref_logprobs", "old_values")
                         if getattr(t, k) is not None}
                    if f:
                        fields[t.request_id] = f
                if fields:
                    cp.post_per_sample(b, fields)
            done = hi
            chunks += 1
            t0 = time.monotonic()
        elif ready:
            if group is not None:
                # every rank has posted before any rank makes the control plane build the batch
                dist.barrier(group=group)
            return chunks
        else:
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"buffer {b}: no progress for the per-sample overlap")
            time.sleep(poll_s)
