"""Hybrid multi-GPU placement: every rank trains AND serves rollout.

N processes, one per GPU (``torch.distributed.run``).  Each rank

* trains: a full bf16 replica of the policy under
  :class:`~psrl_b200.parallel.fsdp.FlatShardedDP` over all N ranks (fp32
  gradients reduce-scattered, sharded AdamW, parameters all-gathered back —
  NCCL over NVLink), on its token-balanced share of every staleness buffer;
* serves rollout: one engine in its own thread on a high-priority stream,
  overlapped with training exactly like the one-GPU colocation (the staleness
  bound makes training on buffer ``b`` while generating later buffers legal);
* syncs weights locally: after the optimizer step that produces version
  ``v + 1`` every rank's parameters equal that version, so its engine pulls
  with one in-HBM copy of the flat parameter buffer.  No weight byte crosses
  NVLink; the only inter-GPU traffic is the gradient reduce-scatter and the
  parameter all-gather of the optimizer step.

The Parameter Server, the dispatcher and the batch planner run in a separate
CPU process (:mod:`.control_plane`); rank 0 starts it.  The process-local
reader-writer lock orders the in-place optimizer update (exclusive) against
the engine's weight copy (shared); the global version is bumped by rank 0 only
after every rank finished its optimizer step, so an engine's version label
never exceeds the weights it holds.

The reference runs trainers and rollout replicas as disjoint Ray resource
pools (``psrl/trainer/main_ppo.py``, ``psrl/trainer/ppo/ray_trainer.py``);
:mod:`.distributed` provides that disaggregated placement, this module the
colocated one scaled out.
"""

from __future__ import annotations

import contextlib
import os
import sys
import time

import torch
import torch.distributed as dist

from ..models import model_args_from_config
from ..parallel import dist as pdist
from ..parallel.weight_sync import WeightLayout
from ..rollout.engine import EngineWeights, RolloutEngine
from ..rollout.instance import SyncPolicy
from ..utils import transfer
from ..utils.locks import RWLock
from ..utils.rpc import RPCClient
from . import algos
from .actor import PolicyWorker
from .control_plane import ExchangeMailbox, spawn_control_plane
from .driver import _apply_switch_interval, train_stream_ctx, trainer_stream_for
from .strategies import (overlap_per_sample, per_sample_missing, pre_step_train, sharded_overlap_enabled,
                         sharded_overlap_mode)


def log(msg: str) -> None:
    r = os.environ.get("RANK", "0")
    print(f"[rank {r} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


class HybridRun:
    def __init__(self, cfg, info: pdist.DistInfo):
        self.cfg = cfg
        self.info = info
        self.rank, self.world = info.rank, info.world_size
        self.device = info.device
        self.is_cuda = self.device.type == "cuda"
        self.args = model_args_from_config(cfg.model)
        self.trained_tokens = 0
        self.global_step = 0
        from ..utils.events import rank_event_log
        self.log = rank_event_log(cfg, self.rank, "hybrid")
        from ..utils.profiling import StepObserver
        self.obs = StepObserver(cfg, self.device, self.rank)
        self.liveness_s = float(cfg.trainer.get("liveness_timeout_s", 300))
        self.buffer_timeout_s = float(cfg.trainer.get("buffer_timeout_s", 1800))
        self.cp_proc = None
        port = 0
        if self.rank == 0:
            self.cp_proc, port = spawn_control_plane(cfg, self.args.vocab_size, self.world, 0, self.liveness_s)
            self.cli_train = RPCClient(("127.0.0.1", port), retries=6000)
            self.cli_train.call("cp", "ping")
        port = pdist.broadcast_value(port)
        if self.rank != 0:
            self.cli_train = RPCClient(("127.0.0.1", port), retries=6000)
        self.cli_roll = RPCClient(("127.0.0.1", port), retries=6000)
        self.cp = self.cli_train.proxy("cp")
        self.cp_roll = self.cli_roll.proxy("cp")
        self.cpu_group = pdist.new_subgroup(list(range(self.world)), backend="gloo") if self.world > 1 else None
        # trainer layout: tensor-parallel groups of `tp` consecutive ranks, data
        # parallelism across them (expert parallelism spans the data-parallel group)
        if int(cfg.actor.get("context_parallel_size", 1) or 1) > 1 or \
                int(cfg.actor.get("ulysses_sequence_parallel_size", 1) or 1) > 1 or \
                int(cfg.actor.get("pipeline_parallel_size", 1) or 1) > 1:
            raise ValueError("context / sequence and pipeline parallelism run in the disaggregated placement")
        tp = int(cfg.actor.get("tensor_parallel_size", 1) or 1)
        if self.world % tp:
            raise ValueError(f"world size {self.world} is not a multiple of tensor_parallel_size={tp}")
        self.tp_size = tp
        self.dp_rank, self.dp_world = self.rank // tp, self.world // tp
        dp_group = tp_group = None
        if self.world > 1:
            if tp == 1:
                dp_group = dist.group.WORLD
            else:
                for k in range(self.dp_world):        # every rank creates every group (same order)
                    g = dist.new_group(list(range(k * tp, (k + 1) * tp)))
                    if k == self.dp_rank:
                        tp_group = g
                for j in range(tp):
                    g = dist.new_group(list(range(j, self.world, tp)))
                    if j == self.rank % tp:
                        dp_group = g
                if self.dp_world == 1:
                    dp_group = None
        seed = int(cfg.trainer.seed)
        self.actor = PolicyWorker(cfg, self.args, self.device, dp_group=dp_group, seed=seed,
                                  dp_rank=self.dp_rank, dp_world=self.dp_world, tp_group=tp_group)
        self.assembler = None
        # rollout TP equal to the trainer's: each engine holds the same shards as its trainer
        rtp = int(cfg.rollout.get("tensor_parallel_size", 1) or 1)
        self.eng_tp = None
        if rtp > 1:
            if self.actor.tp is None or rtp != tp or self.actor.ep is not None:
                raise ValueError("rollout.tensor_parallel_size > 1 needs the same actor.tensor_parallel_size")
            from ..parallel.tp import make_tp_group
            k = self.dp_rank
            ranks = list(range(k * tp, (k + 1) * tp))
            # separate communicators: the engine's all-reduces run on the rollout thread
            eng_groups = [dist.new_group(list(range(j * tp, (j + 1) * tp))) for j in range(self.dp_world)]
            cpu_groups = [dist.new_group(list(range(j * tp, (j + 1) * tp)), backend="gloo")
                          for j in range(self.dp_world)]
            self.eng_tp = make_tp_group(eng_groups[k])
            self.eng_tp_cpu = cpu_groups[k]
            self.eng_leader = ranks[0]
        elif self.actor.ep is not None or self.actor.tp is not None:
            # the engine holds the full model; sharded weights are all-gathered after each step
            from ..parallel.assemble import FullWeightAssembler
            self.assembler = FullWeightAssembler(
                self.actor.model, ep=self.actor.ep, tp=self.actor.tp,
                ep_names=[n for n in dict(self.actor.model.named_parameters()) if "experts_w" in n]
                if self.actor.ep is not None else (),
                tp_names=sorted(self.actor.tp_sharded) if self.actor.tp is not None else ())
        self.critic = None
        if cfg.critic.enable:
            from dataclasses import replace as _replace
            cargs = _replace(self.args, value_head=True, tie_word_embeddings=False)
            self.critic = PolicyWorker(cfg, cargs, self.device, dp_group=dp_group, seed=seed + 1,
                                       dp_rank=self.dp_rank, dp_world=self.dp_world, tp_group=tp_group)
        self.ref = None
        if cfg.actor.use_kl_loss or cfg.algorithm.use_kl_in_reward:
            # sharded like the actor (expert / tensor parallel forwards are collectives)
            self.ref = PolicyWorker(cfg, self.args, self.device, dp_group=dp_group, seed=seed, trainable=False,
                                    dp_rank=self.dp_rank, dp_world=self.dp_world, tp_group=tp_group)
        self.kl_ctrl = algos.kl_controller(cfg.algorithm) if cfg.algorithm.use_kl_in_reward else None
        # resume: the control plane already re-seated the data cursor and the PS
        # version; every rank loads its part before the engine copies its weights
        self.resumed = self.cp.resumed_step()
        if self.resumed is not None:
            from ..utils.checkpoint import load_trainer_ranks
            root = cfg.trainer.get("resume_from_path") or cfg.trainer.default_local_dir
            extra = load_trainer_ranks(root, self.resumed, self.actor, self.critic, self.rank,
                                       bool(cfg.psrl.checkpoint.use_dcp_save))
            if self.kl_ctrl is not None and "kl_coef" in extra:
                self.kl_ctrl.value = float(extra["kl_coef"])
            self.global_step = self.resumed
        self.sharded_overlap = sharded_overlap_enabled(cfg)
        self.pre_step = sharded_overlap_mode(cfg) == "pre_step"
        self.wlock = RWLock()
        self.eng_sources = None
        if self.eng_tp is not None:
            # engine weights: copies of this rank's trainer shards (engine names)
            from ..parallel.assemble import engine_name
            w = EngineWeights(self.args, self.device, self.actor.dtype)
            self.eng_sources = []
            for n, p in self.actor.model.named_parameters():
                t = p.detach().clone()
                w.tensors[engine_name(n)] = t
                self.eng_sources.append((t, p))
            for name, b in self.actor.model.named_buffers():
                w.tensors[name] = b.to(self.device)
            self.eng_flat = None
        elif self.assembler is None:
            # engine weights: one flat copy in the trainer's flat layout (a pull is one copy)
            layout = WeightLayout.from_dp(self.actor.dp)
            self.eng_flat = self.actor.dp.flat.detach().clone()
            w = EngineWeights(self.args, self.device, self.actor.dtype)
            w.flat = self.eng_flat
            w.tensors = layout.views(self.eng_flat)
            for name, b in self.actor.model.named_buffers():
                w.tensors[name] = b.to(self.device)
        else:
            # engine weights: the full (unsharded) model, filled by the assembler
            from ..models import build_model
            full = build_model(self.args, self.device, self.actor.dtype, seed=seed)
            w = EngineWeights.from_model(full, self.device, dtype=self.actor.dtype)
            del full
            self.eng_flat = None
            with self.wlock.exclusive(600):
                self.assembler.gather()
                self.assembler.assemble_into(w.tensors)
        self.engine_weights = w
        rc = cfg.rollout
        max_len = int(rc.max_prompt_length) + int(rc.max_response_length) + 64
        self.engine = RolloutEngine(
            self.args, w, max_num_seqs=int(rc.max_num_seqs), max_model_len=max_len, block_size=int(rc.block_size),
            max_num_batched_tokens=int(rc.max_num_batched_tokens), kv_cache_gb=float(rc.get("kv_cache_gb", 4.0)),
            enable_prefix_caching=bool(rc.enable_prefix_caching), use_cuda_graph=bool(rc.cuda_graph),
            keep_kv_on_update=bool(cfg.psrl.rollout_coordination.partial_rollout.get("keep_kv", False)),
            eos_token_id=None if rc.ignore_eos else self.cp.eos_id(), tp=self.eng_tp, decode_gemm=str(cfg.rollout.get("decode_gemm", "library")),
            kv_offload_blocks=int(cfg.rollout.get("kv_offload_blocks", 0) or 0))
        sm = cfg.psrl.rollout_coordination.sync_and_mig_strategy
        self.policy = SyncPolicy(sm.method, bool(cfg.psrl.rollout_coordination.partial_rollout.enable),
                                 sm.sync.get("threshold"), sm.sync.get("indicator", "request_num"))
        # one rollout instance per engine; a TP engine's instance is its leader's
        self.is_leader = self.eng_tp is None or self.rank == self.eng_leader
        self.instance_id = (self.rank if self.eng_tp is None else self.eng_leader, 0)
        if self.is_leader:
            self.cp.register_instance(self.instance_id, self.engine.version)
        self.rollout_stream = torch.cuda.Stream(device=self.device, priority=-1) if self.is_cuda else None
        self.train_stream = trainer_stream_for(cfg, self.device, self.is_cuda)
        _apply_switch_interval(cfg)
        self.mailbox: ExchangeMailbox | None = None
        self._thread = None
        self._stop = False
        self._rollout_error: BaseException | None = None
        self.pulls = 0
        self.pull_s = 0.0
        log(f"hybrid rank ready: trainer dp{self.world} + rollout instance {self.instance_id}")

    def _save_checkpoint(self) -> None:
        """Every rank saves its part of ``global_step`` (under the shared weight
        lock, so no optimizer step runs meanwhile); rank 0 then adds the control
        plane's data cursor and marks the step complete."""
        from ..utils.checkpoint import finish_trainer_checkpoint, save_trainer_ranks
        cfg = self.cfg
        root = cfg.trainer.default_local_dir
        with self.wlock.shared(600):
            save_trainer_ranks(root, self.global_step, self.actor, self.critic, self.rank, None,
                               bool(cfg.psrl.checkpoint.use_dcp_save))
        if self.cpu_group is not None:
            dist.barrier(group=self.cpu_group)
        if self.rank == 0:
            extra = {"kl_coef": self.kl_ctrl.value} if self.kl_ctrl is not None else {}
            finish_trainer_checkpoint(root, self.global_step, self.cp.checkpoint_meta(), extra)

    # -------------------------------------------------------------- rollout
    def _pull(self, v: int | None = None) -> None:
        """Refresh the engine from the local trainer.  ``v``: the version a TP
        leader already read (followers take it from the leader's broadcast)."""
        t0 = time.perf_counter()
        with self.wlock.shared(600):
            # the PS version is read first: the local parameters are at least that new
            if v is None:
                v = self.cp_roll.pull_model(self.instance_id)
            if self.eng_sources is not None:
                for t, p in self.eng_sources:
                    t.copy_(p.detach(), non_blocking=True)
            elif self.assembler is None:
                self.eng_flat.copy_(self.actor.dp.flat, non_blocking=True)
            else:
                self.assembler.assemble_into(self.engine_weights.tensors)
            if self.is_cuda:
                torch.cuda.current_stream().synchronize()
        self.engine.load_weights(None, v)
        dt = time.perf_counter() - t0
        self.pulls += 1
        self.pull_s += dt
        self.log.record_span("PULL", time.time() - dt, dt, version=int(v))
        if self.is_leader:
            self.cp_roll.report_pull(dt)

    def _tp_rollout_loop(self) -> None:
        """TP engine: the leader talks to the control plane and broadcasts each
        round's requests, aborts, weight version and stop flag to its followers,
        so every TP rank applies identical operations and steps in lockstep."""
        eng = self.engine
        mb = self.mailbox
        leader = self.is_leader
        try:
            ctx = torch.cuda.stream(self.rollout_stream) if self.is_cuda else contextlib.nullcontext()
            with ctx:
                while True:
                    msg = None
                    if leader:
                        reqs, aborts = mb.collect()
                        v = None
                        if self.policy.should_sync(eng, mb.ps_version):
                            v = self.cp_roll.pull_model(self.instance_id)
                        msg = (reqs, aborts, v, bool(self._stop))
                    box = [msg]
                    dist.broadcast_object_list(box, src=self.eng_leader, group=self.eng_tp_cpu)
                    reqs, aborts, v, stop = box[0]
                    if stop:
                        break
                    for r in reqs:
                        eng.add_request(r)
                    for rid in aborts:
                        eng.abort(rid)
                    if v is not None:
                        self._pull(v)
                    if eng.has_unfinished():
                        outs = eng.step()
                        if outs and leader:
                            mb.post(outs)
                    else:
                        if leader:
                            mb.kick()
                        time.sleep(0.0005)
        except BaseException as exc:
            self._rollout_error = exc
            if leader:
                with contextlib.suppress(Exception):
                    self.cp_roll.report_failure(self.instance_id, f"{type(exc).__name__}: {exc}")

    def _rollout_loop(self) -> None:
        if self.eng_tp is not None:
            return self._tp_rollout_loop()
        eng = self.engine
        mb = self.mailbox
        try:
            ctx = torch.cuda.stream(self.rollout_stream) if self.is_cuda else contextlib.nullcontext()
            with ctx:
                while not self._stop:
                    reqs, aborts = mb.collect()
                    for r in reqs:
                        eng.add_request(r)
                    for rid in aborts:
                        eng.abort(rid)
                    if self.policy.should_sync(eng, mb.ps_version):
                        self._pull()
                    if eng.has_unfinished():
                        outs = eng.step()
                        if outs:
                            mb.post(outs)
                    else:
                        mb.kick()
                        time.sleep(0.0005)
        except BaseException as exc:    # surfaced to the trainer thread and the control plane
            self._rollout_error = exc
            with contextlib.suppress(Exception):
                self.cp_roll.report_failure(self.instance_id, f"{type(exc).__name__}: {exc}")

    def start_rollout(self) -> None:
        if self._thread is None:
            import threading
            self._stop = False
            if self.is_leader:
                self.mailbox = ExchangeMailbox(self.cp_roll, self.instance_id, self.engine)
            self._thread = threading.Thread(target=self._rollout_loop, daemon=True, name="rollout")
            self._thread.start()

    def stop_rollout(self) -> None:
        if self._thread is not None:
            self._stop = True
            self._thread.join()
            self._thread = None
        if self.mailbox is not None:
            self.mailbox.close()
            self.mailbox = None

    # -------------------------------------------------------------- training
    def step(self) -> dict:
        b = self.global_step
        self.obs.begin(b)
        if self._rollout_error is not None:
            raise RuntimeError("rollout thread failed") from self._rollout_error
        self.start_rollout()
        t0 = time.perf_counter()
        chunks = 0
        if self.sharded_overlap:
            with train_stream_ctx(self.train_stream):
                chunks = overlap_per_sample(
                    self.cfg, self.cp, b, lambda ts: per_sample_missing(self.cfg, ts, self.actor, self.ref, self.critic),
                    group=self.cpu_group, src=0, dp_rank=self.dp_rank, dp_world=self.dp_world,
                    post=self.rank % self.tp_size == 0, timeout_s=self.buffer_timeout_s)
        pre_metrics = None
        if self.pre_step:
            # train each committed mini-batch as it arrives; the batch below is only consumed
            with train_stream_ctx(self.train_stream):
                pre_metrics, chunks = pre_step_train(
                    self.cfg, self.cp, b, self.actor, self.ref, group=self.cpu_group, src=0, dp_rank=self.dp_rank,
                    dp_world=self.dp_world, step_guard=lambda: self.wlock.exclusive(600),
                    sync_every_micro_batch=self.is_cuda, timeout_s=self.buffer_timeout_s)
        batch = self.cp.get_batch(b, self.dp_rank, self.dp_world, self.buffer_timeout_s, self.rank % self.tp_size,
                                  self.tp_size)
        trajs, plan = batch["trajs"], batch["plan"]
        t1 = time.perf_counter()
        pre = sum(1 for t in trajs if t.ref_logprobs is not None or t.old_values is not None
                  or (t.old_logprobs is not None and t.old_logprobs is not t.rollout_logprobs))
        with train_stream_ctx(self.train_stream):
            if pre_metrics is not None:
                metrics, critic_metrics = dict(pre_metrics), {}
            else:
                per_sample_missing(self.cfg, trajs, self.actor, self.ref, self.critic)
                critic_metrics = algos.shard_advantages(self.cfg, trajs, self.cpu_group, self.kl_ctrl, self.tp_size,
                                                        critic=self.critic is not None)
                critic_metrics.update(algos.apply_rollout_correction(self.cfg.algorithm.rollout_correction, trajs))
                if self.critic is not None:
                    critic_metrics.update(self.critic.update_critic(trajs, plan=plan))
                metrics = self.actor.update_policy(trajs, float(self.cfg.rollout.temperature),
                                                   step_guard=lambda: self.wlock.exclusive(600),
                                                   sync_every_micro_batch=self.is_cuda, plan=plan)
            if self.assembler is not None:
                # all ranks: gather the sharded weights for the full-model engines
                with self.wlock.exclusive(600):
                    self.assembler.gather()
                    if self.is_cuda:
                        torch.cuda.current_stream().synchronize()
        t2 = time.perf_counter()
        if self.cpu_group is not None:
            dist.barrier(group=self.cpu_group)      # every replica holds version b + 1
        if self.rank == 0:
            self.cp.push_model(b + 1)
        self.global_step += 1
        self.trained_tokens += int(batch["trained_tokens"])
        metrics.update(batch["metrics"])
        metrics.update(critic_metrics)
        metrics.update({
            "step": b, "num_trajectories": batch["num_trajectories"], "trained_tokens": batch["trained_tokens"],
            "response_length/mean": batch["response_length/mean"], "staleness/max": batch["staleness/max"],
            "timing_s/gen_wait": t1 - t0, "timing_s/train": t2 - t1, "timing_s/step": time.perf_counter() - t0,
            "rollout/pulls": self.pulls, "rollout/pull_s": self.pull_s, "fine_grain/chunks": chunks,
            "fine_grain/precomputed": pre,
        })
        metrics.update({f"rollout/{k}": v for k, v in self.engine.engine_stats().items() if isinstance(v, (int, float))})
        from .perf import perf_metrics
        metrics.update(perf_metrics(self.cfg, self.args, int(batch["trained_tokens"]), int(batch["num_trajectories"]),
                                    metrics["timing_s/step"], t2 - t1, self.world, self.world))
        from .distributed import _log_step_spans
        _log_step_spans(self.log, b, t0, t1, t2, metrics)
        self.obs.end(b, metrics)
        sf = int(self.cfg.trainer.get("save_freq", -1) or -1)
        if sf > 0 and self.global_step % sf == 0:
            t3 = time.perf_counter()
            self._save_checkpoint()
            metrics["timing_s/checkpoint"] = time.perf_counter() - t3
        tf = int(self.cfg.trainer.get("test_freq", -1) or -1)
        if tf > 0 and self.global_step % tf == 0 and self.rank == 0:
            # validation on the rollout instances with the weights just pushed
            t3 = time.perf_counter()
            metrics.update(self.cp.validate())
            metrics["timing_s/validate"] = time.perf_counter() - t3
        return metrics

    def close(self) -> None:
        self.stop_rollout()
        if self.rank == 0:
            with contextlib.suppress(Exception):
                self.cp.shutdown()
        for c in (self.cli_roll, self.cli_train):
            c.close()
        if self.cp_proc is not None:
            self.cp_proc.join(timeout=30)
            if self.cp_proc.is_alive():
                self.cp_proc.terminate()


def run_hybrid(cfg, steps: int, warmup: int, info: pdist.DistInfo | None = None, capture: bool = True) -> dict:
    """``warmup`` + ``steps`` training steps on every rank; returns the timing
    (max over ranks) and, on rank 0, metrics, token counts and control-plane stats."""
    info = info or pdist.init_distributed(cfg.trainer.get("device", "auto"))
    run = HybridRun(cfg, info)
    if steps is None:
        # trainer.total_training_steps counts from step 0 (a resumed run does the rest)
        steps = max(0, int(cfg.trainer.total_training_steps) - int(getattr(run, "global_step", 0)))
    is_cuda = info.device.type == "cuda"
    if capture and is_cuda and run.engine.use_cuda_graph:
        run.engine.capture_all()
    t_evt: dict = {}

    def mark(p):
        pdist.barrier()
        if is_cuda:
            torch.cuda.synchronize()
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            t_evt[p] = ev
        t_evt[f"wall{p}"] = time.perf_counter()
        t_evt[f"xfer{p}"] = transfer.snapshot()

    metrics = []
    try:
        for i in range(warmup):
            m = run.step()
            if run.rank == 0:
                log(f"warm-up step {i}: {m['timing_s/step']:.1f}s (wait {m['timing_s/gen_wait']:.1f}s), "
                    f"{m['trained_tokens']} tokens")
        mark(1)
        for i in range(steps):
            metrics.append(run.step())
            if run.rank == 0:
                m = metrics[-1]
                log(f"timed step {i}: {m['timing_s/step']:.1f}s (wait {m['timing_s/gen_wait']:.1f}s), "
                    f"{m['trained_tokens']} tokens")
        mark(2)
        if is_cuda:
            torch.cuda.synchronize()
            ms = t_evt[1].elapsed_time(t_evt[2])
        else:
            ms = (t_evt["wall2"] - t_evt["wall1"]) * 1000.0
        wall = t_evt["wall2"] - t_evt["wall1"]
        # host<->device bytes of this rank inside the timed region
        xfer = [b - a for a, b in zip(t_evt["xfer1"], t_evt["xfer2"])]
        run.stop_rollout()
        ms_max = pdist.all_reduce_max(ms, info.device)
        wall_max = pdist.all_reduce_max(wall, info.device)
        out = {"ms": ms_max, "wall_s": wall_max, "rank": run.rank, "metrics": metrics, "world": run.world,
               "h2d": xfer[0], "d2h": xfer[1],
               "tokens": sum(int(m["trained_tokens"]) for m in metrics),
               "param_checksum": float(run.actor.dp.flat.double().sum()),
               "engine_checksum": float(sum(t.double().sum() for k, t in run.engine_weights.tensors.items()
                                            if "prior" not in k))}
        if run.rank == 0:
            out["cp"] = run.cp.stats()
        pdist.barrier()
    finally:
        run.close()
    return out
