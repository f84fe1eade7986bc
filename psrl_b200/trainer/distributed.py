"""Disaggregated asynchronous RL over N processes (one per device).

Ranks ``[0, T)`` train (sharded data parallel over an NCCL group), ranks
``[T, N)`` each run one rollout instance.  The Parameter Server, the
dispatcher (agent-loop manager, reward) and the batch planner run in a CPU
control-plane process started by rank 0 (:mod:`.control_plane`); rollout ranks
talk to it through an asynchronous exchange mailbox (trajectories travel back
in the same RPC that fetches new work, which replaces the reference's Ray
actors, the SMG router's gRPC admission calls and the TransferQueue hop), and
each trainer rank fetches only its own token-balanced share of a buffer.

Weights: every trainer rank publishes its parameters into its
:class:`~psrl_b200.parallel.weight_sync.WeightStore` (HBM) under the PS
exclusive-push lock; rollout ranks pull slices from all trainers over NVLink
under the shared-pull lock whenever their sync policy allows.

On CPU the same code runs with gloo and a shared-memory store (the
world_size=2 plumbing configuration).
"""

from __future__ import annotations

import contextlib
import os
import sys
import time

import torch
import torch.distributed as dist

from ..models import model_args_from_config
from ..models.qwen import zipf_prior
from ..parallel import dist as pdist
from ..parallel.weight_sync import ShardedWeightPuller, WeightLayout, WeightPuller, WeightStore
from ..rollout.engine import EngineWeights, RolloutEngine
from ..rollout.instance import SyncPolicy
from ..utils import transfer
from ..utils.rpc import RPCClient
from . import algos
from .actor import PolicyWorker
from .control_plane import ExchangeMailbox, spawn_control_plane
from .strategies import (overlap_per_sample, per_sample_missing, pre_step_train, sharded_overlap_enabled,
                         sharded_overlap_mode)


def log(msg: str) -> None:
    r = os.environ.get("RANK", "0")
    print(f"[rank {r} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def _role_split(world: int, cfg) -> int:
    t = int(cfg.psrl.deployment.get("train_ngpus", 0) or 0)
    if t <= 0 or t >= world:
        t = max(1, world // 2)
    return t


def full_model_layout(args, dtype) -> WeightLayout:
    """Flat layout of the unsharded model's parameters (each tensor 64-element
    aligned), the layout rollout engines hold their weights in."""
    from ..models.qwen import QwenModel
    with torch.device("meta"):
        shapes = [(n, tuple(p.shape)) for n, p in QwenModel(args).named_parameters()]
    entries, off = [], 0
    for n, shp in shapes:
        entries.append((n, shp, off))
        k = 1
        for d in shp:
            k *= d
        off += (k + 63) // 64 * 64
    return WeightLayout(entries, off, dtype)


class DisaggregatedRun:
    def __init__(self, cfg, info: pdist.DistInfo):
        self.cfg = cfg
        self.info = info
        self.world = info.world_size
        self.rank = info.rank
        self.n_train = _role_split(self.world, cfg)
        self.is_trainer = self.rank < self.n_train
        self.device = info.device
        trainer_ranks = list(range(self.n_train))
        backend = "nccl" if self.device.type == "cuda" else "gloo"
        self.train_group = None
        self.train_cpu_group = None
        # trainer layout: tensor-parallel groups of `tp` consecutive trainer ranks,
        # data parallelism across them
        # sizes: this framework's keys, or the reference's Megatron-backend names
        meg = cfg.actor.get("megatron", None) or {}
        tp = max(int(cfg.actor.get("tensor_parallel_size", 1) or 1), int(meg.get("tensor_model_parallel_size", 1) or 1))
        cpn = max(int(cfg.actor.get("context_parallel_size", 1) or 1), int(meg.get("context_parallel_size", 1) or 1))
        # Ulysses sequence parallelism (veRL's name) takes the context-parallel groups
        usp = int(cfg.actor.get("ulysses_sequence_parallel_size", 1) or 1)
        self.cp_mode = "zigzag"
        if usp > 1:
            if cpn > 1:
                raise ValueError("context parallelism and Ulysses sequence parallelism are alternatives; set one")
            cpn, self.cp_mode = usp, "ulysses"
        ppn = max(int(cfg.actor.get("pipeline_parallel_size", 1) or 1),
                  int(meg.get("pipeline_model_parallel_size", 1) or 1))
        if sum(x > 1 for x in (tp, cpn, ppn)) > 1:
            raise ValueError("tensor, context and pipeline parallelism combine with data parallelism only, "
                             "not with each other")
        gsize = tp * cpn * ppn
        if self.n_train % gsize:
            raise ValueError(f"{self.n_train} trainer ranks are not a multiple of the model-parallel size {gsize}")
        # ranks of one TP / CP / PP group hold the same data share
        self.tp_size = gsize
        self.dp_rank, self.dp_world = self.rank // gsize, self.n_train // gsize
        self.tp_group = self.cp_group = self.pp_group = None
        self.pp_size = ppn
        if self.is_trainer and self.n_train > 1:
            # created by the trainer ranks only (group-local synchronisation)
            self.train_cpu_group = pdist.new_subgroup(trainer_ranks, backend="gloo")
            if gsize == 1 or cpn > 1:
                # data (and context) parallel gradients sum over every trainer rank
                self.train_group = pdist.new_subgroup(trainer_ranks, backend=backend)
            if gsize > 1:
                for k in range(self.dp_world):
                    g = pdist.new_subgroup(list(range(k * gsize, (k + 1) * gsize)), backend=backend) \
                        if k == self.dp_rank else None
                    if g is not None:
                        if tp > 1:
                            self.tp_group = g
                        elif cpn > 1:
                            self.cp_group = g
                        else:
                            self.pp_group = g
                if cpn == 1 and self.dp_world > 1:
                    # TP shard / PP stage j of every replica reduce their gradients together
                    self.train_group = pdist.new_subgroup(list(range(self.rank % gsize, self.n_train, gsize)),
                                                          backend=backend)
        self.args = model_args_from_config(cfg.model)
        # tensor-parallel rollout engines: groups of `rtp` consecutive rollout
        # ranks serve one instance; the first rank of a group (the leader)
        # talks to the control plane and broadcasts every round to the others
        # (heterogeneous instances: rollout.tensor_parallel_sizes lists one TP size
        # per instance, in rollout-rank order)
        n_roll = self.world - self.n_train
        sizes = list(cfg.rollout.get("tensor_parallel_sizes", None) or [])
        if sizes:
            sizes = [int(x) for x in sizes]
            if sum(sizes) != n_roll or min(sizes) < 1:
                raise ValueError(f"rollout.tensor_parallel_sizes {sizes} must add up to the {n_roll} rollout ranks")
        else:
            rtp = int(cfg.rollout.get("tensor_parallel_size", 1) or 1)
            if n_roll % rtp:
                raise ValueError(f"{n_roll} rollout ranks are not a multiple of rollout.tensor_parallel_size {rtp}")
            sizes = [rtp] * (n_roll // rtp)
        self.rollout_tp_sizes = sizes
        self.eng_tp = self.eng_tp_cpu = None
        self.eng_leader = self.rank
        if not self.is_trainer:
            start = self.n_train
            for sz in sizes:
                if start <= self.rank < start + sz and sz > 1:
                    from ..parallel.tp import make_tp_group
                    ranks = list(range(start, start + sz))
                    self.eng_tp = make_tp_group(pdist.new_subgroup(ranks, backend=backend))
                    self.eng_tp_cpu = pdist.new_subgroup(ranks, backend="gloo")
                    self.eng_leader = ranks[0]
                start += sz
        self.is_leader = self.eng_tp is None or self.rank == self.eng_leader
        self.trained_tokens = 0
        self.global_step = 0
        from ..utils.events import rank_event_log
        self.log = rank_event_log(cfg, self.rank, "trainer" if self.is_trainer else "rollout")
        from ..utils.profiling import StepObserver
        self.obs = StepObserver(cfg, self.device, self.rank)
        self.liveness_s = float(cfg.trainer.get("liveness_timeout_s", 300))
        self.buffer_timeout_s = float(cfg.trainer.get("buffer_timeout_s", 1800))
        log(f"role split: {self.n_train} trainer rank(s), {self.world - self.n_train} rollout rank(s)")
        self.cp_proc = None
        port = 0
        if self.rank == 0:
            self.cp_proc, port = spawn_control_plane(cfg, self.args.vocab_size, self.n_train, 0, self.liveness_s)
            self.client = RPCClient(("127.0.0.1", port), retries=6000)
            self.client.call("cp", "ping")
        port = pdist.broadcast_value(port)
        if self.rank != 0:
            self.client = RPCClient(("127.0.0.1", port), retries=6000)
        self.cp = self.client.proxy("cp")
        log("control plane up")
        self.mailbox = None
        if self.is_trainer:
            self._init_trainer()
        else:
            self._init_rollout()

    # ------------------------------------------------------------ trainer
    def _init_trainer(self):
        cfg = self.cfg
        self.actor = PolicyWorker(cfg, self.args, self.device, dp_group=self.train_group,
                                  seed=int(cfg.trainer.seed), dp_rank=self.dp_rank, dp_world=self.dp_world,
                                  tp_group=self.tp_group, cp_group=self.cp_group, cp_mode=self.cp_mode,
                                  pp_group=self.pp_group)
        self.assembler = None
        self.pub_parts = None
        if self.actor.tp is not None and self.actor.ep is None:
            # tensor-parallel trainer: each rank publishes its own shards (replicated
            # parameters, then sharded ones); rollout ranks put the full tensors
            # together while they pull (parallel.weight_sync.ShardedWeightPuller)
            dp, dpp = self.actor.dp, self.actor.dp_partner
            entries = list(dp.layout) + [(n, shp, dp.total + off) for n, shp, off in dpp.layout]
            self.layout = WeightLayout(entries, dp.total + dpp.total, self.actor.dtype)
            self.pub_parts = [dp.flat, dpp.flat]
            self.pub_flat = None
        elif self.actor.ep is not None or self.actor.tp is not None:
            # sharded trainer: every trainer rank publishes the full model, assembled
            # from the shards after each optimizer step (rollout ranks pull as usual)
            from ..parallel.assemble import FullWeightAssembler
            m = self.actor.model
            self.assembler = FullWeightAssembler(
                m, ep=self.actor.ep, tp=self.actor.tp,
                ep_names=[n for n, _ in m.named_parameters() if "experts_w" in n] if self.actor.ep is not None else (),
                tp_names=sorted(self.actor.tp_sharded) if self.actor.tp is not None else ())
            self.layout = full_model_layout(self.args, self.actor.dtype)
            self.pub_flat = torch.zeros(self.layout.total, dtype=self.actor.dtype, device=self.device)
            self.pub_views = self.layout.views(self.pub_flat)
            self.assembler.gather()
            self.assembler.assemble_into(self.pub_views)
        else:
            self.layout = WeightLayout.from_dp(self.actor.dp)
            self.pub_flat = self.actor.dp.flat
        self.critic = None
        if cfg.critic.enable:
            from dataclasses import replace as _replace
            cargs = _replace(self.args, value_head=True, tie_word_embeddings=False)
            self.critic = PolicyWorker(cfg, cargs, self.device, dp_group=self.train_group,
                                       seed=int(cfg.trainer.seed) + 1, dp_rank=self.dp_rank, dp_world=self.dp_world,
                                       tp_group=self.tp_group, cp_group=self.cp_group, cp_mode=self.cp_mode,
                                       pp_group=self.pp_group)
        self.ref = None
        if cfg.actor.use_kl_loss or cfg.algorithm.use_kl_in_reward:
            # sharded like the actor (expert / tensor parallel forwards are collectives)
            self.ref = PolicyWorker(cfg, self.args, self.device, dp_group=self.train_group,
                                    seed=int(cfg.trainer.seed), trainable=False, dp_rank=self.dp_rank,
                                    dp_world=self.dp_world, tp_group=self.tp_group, cp_group=self.cp_group, cp_mode=self.cp_mode,
                                    pp_group=self.pp_group)
        self.kl_ctrl = algos.kl_controller(cfg.algorithm) if cfg.algorithm.use_kl_in_reward else None
        self.sharded_overlap = sharded_overlap_enabled(cfg)
        self.pre_step = sharded_overlap_mode(cfg) == "pre_step"
        mode = "hbm" if (cfg.psrl.ps_mode == "hbm" and self.device.type == "cuda") else "cpu"
        self.store = WeightStore(self.layout, self.device, mode)
        # resume: the control plane already re-seated the data cursor and the PS
        # version; every trainer rank loads its part of the same step
        self.resumed = self.cp.resumed_step()
        if self.resumed is not None:
            from ..utils.checkpoint import load_trainer_ranks
            root = cfg.trainer.get("resume_from_path") or cfg.trainer.default_local_dir
            extra = load_trainer_ranks(root, self.resumed, self.actor, self.critic, self.rank,
                                       bool(cfg.psrl.checkpoint.use_dcp_save), self._ckpt_group())
            if self.kl_ctrl is not None and "kl_coef" in extra:
                self.kl_ctrl.value = float(extra["kl_coef"])
            self.global_step = self.resumed
            log(f"trainer rank {self.rank}: resumed from step {self.resumed}")
        self._publish(self.resumed or 0)
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        desc = self.store.descriptor()
        engine_layout = self.layout
        if self.pub_parts is not None:
            desc.update(entries=list(self.layout.entries), tp_rank=self.actor.tp.rank, tp_world=self.actor.tp.world)
            engine_layout = full_model_layout(self.args, self.actor.dtype)
        if self.pp_size > 1:
            # each stage publishes its own layers; rollout ranks pull every tensor from a
            # stage that holds it, straight into the full engine layout
            desc["entries"] = list(self.layout.entries)
            engine_layout = full_model_layout(self.args, self.actor.dtype)
        if self.rank == 0:
            self.cp.set_layout(engine_layout)
        self.cp.register_store(self.rank, desc)
        log(f"trainer ready: {self.layout.nbytes / 2**30:.2f} GiB published store ({mode})")

    def _ckpt_group(self):
        """The trainer ranks' gloo group (DCP must not wait for rollout ranks)."""
        if self.train_cpu_group is not None:
            return self.train_cpu_group
        if getattr(self, "_solo_group", None) is None and dist.is_initialized():
            self._solo_group = pdist.new_subgroup([self.rank], backend="gloo")
        return getattr(self, "_solo_group", None)

    def _save_checkpoint(self) -> None:
        """Every trainer rank saves its part of ``global_step``; rank 0 then
        adds the control plane's data cursor and marks the step complete."""
        from ..utils.checkpoint import finish_trainer_checkpoint, save_trainer_ranks
        cfg = self.cfg
        root = cfg.trainer.default_local_dir
        save_trainer_ranks(root, self.global_step, self.actor, self.critic, self.rank, None,
                           bool(cfg.psrl.checkpoint.use_dcp_save), group=self._ckpt_group())
        if self.n_train > 1:
            dist.barrier(group=self.train_cpu_group)
        if self.rank == 0:
            extra = {"kl_coef": self.kl_ctrl.value} if self.kl_ctrl is not None else {}
            finish_trainer_checkpoint(root, self.global_step, self.cp.checkpoint_meta(), extra)

    def _publish(self, version: int) -> None:
        if self.pub_parts is not None:
            self.store.publish_parts(self.pub_parts, version)
        else:
            self.store.publish(self.pub_flat, version)

    def trainer_step(self) -> dict:
        b = self.global_step
        self.obs.begin(b)
        t0 = time.perf_counter()
        chunks = 0
        if self.sharded_overlap:
            chunks = overlap_per_sample(
                self.cfg, self.cp, b, lambda ts: per_sample_missing(self.cfg, ts, self.actor, self.ref, self.critic),
                group=self.train_cpu_group, src=0, dp_rank=self.dp_rank, dp_world=self.dp_world,
                post=self.rank % self.tp_size == 0, timeout_s=self.buffer_timeout_s)
        pre_metrics = None
        if self.pre_step:
            # train each committed mini-batch as it arrives; the batch below is only consumed
            pre_metrics, chunks = pre_step_train(
                self.cfg, self.cp, b, self.actor, self.ref, group=self.train_cpu_group, src=0, dp_rank=self.dp_rank,
                dp_world=self.dp_world, timeout_s=self.buffer_timeout_s)
        batch = self.cp.get_batch(b, self.dp_rank, self.dp_world, self.buffer_timeout_s, self.rank % self.tp_size,
                                  self.tp_size)
        trajs, plan = batch["trajs"], batch["plan"]
        t1 = time.perf_counter()
        pre = sum(1 for t in trajs if t.ref_logprobs is not None or t.old_values is not None
                  or (t.old_logprobs is not None and t.old_logprobs is not t.rollout_logprobs))
        if pre_metrics is not None:
            metrics, critic_metrics = dict(pre_metrics), {}
        else:
            per_sample_missing(self.cfg, trajs, self.actor, self.ref, self.critic)
            critic_metrics = algos.shard_advantages(self.cfg, trajs, self.train_cpu_group, self.kl_ctrl,
                                                    self.tp_size, critic=self.critic is not None)
            critic_metrics.update(algos.apply_rollout_correction(self.cfg.algorithm.rollout_correction, trajs))
            if self.critic is not None:
                critic_metrics.update(self.critic.update_critic(trajs, plan=plan))
            metrics = self.actor.update_policy(trajs, float(self.cfg.rollout.temperature), plan=plan)
        metrics.update(critic_metrics)
        if self.assembler is not None:
            self.assembler.gather()                  # collective over the trainer shards
            self.assembler.assemble_into(self.pub_views)
        t2 = time.perf_counter()
        # publish: PS exclusive lock -> every trainer writes its store -> version bump
        if self.rank == 0 and not self.cp.acquire_push(600):
            raise TimeoutError("exclusive push lock")
        if self.n_train > 1:
            dist.barrier(group=self.train_cpu_group)
        self._publish(b + 1)
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        if self.n_train > 1:
            dist.barrier(group=self.train_cpu_group)
        if self.rank == 0:
            try:
                self.cp.push_model(b + 1, True)
            finally:
                self.cp.release_push()
        self.global_step += 1
        self.trained_tokens += int(batch["trained_tokens"])
        metrics.update(batch["metrics"])
        metrics.update({"step": b, "trained_tokens": batch["trained_tokens"], "fine_grain/chunks": chunks,
                        "fine_grain/precomputed": pre,
                        "num_trajectories": batch["num_trajectories"],
                        "response_length/mean": batch["response_length/mean"],
                        "staleness/max": batch["staleness/max"],
                        "timing_s/gen_wait": t1 - t0, "timing_s/train": t2 - t1,
                        "timing_s/publish": time.perf_counter() - t2,
                        "timing_s/step": time.perf_counter() - t0})
        from .perf import perf_metrics
        metrics.update(perf_metrics(self.cfg, self.args, int(batch["trained_tokens"]),
                                    int(batch["num_trajectories"]), metrics["timing_s/step"], t2 - t1,
                                    self.world, self.n_train))
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

    # ------------------------------------------------------------ rollout
    def _init_rollout(self):
        cfg, a = self.cfg, self.args
        rc = cfg.rollout
        self.instance_id = (self.eng_leader - self.n_train, 0)
        log("rollout: waiting for trainer stores")
        layout, descs = self.cp.get_stores()
        self.layout = layout
        dtype = layout.dtype
        # a TP instance pulls its shards directly from whole-tensor stores, or from a
        # dense TP trainer's stores of the same TP size (rank r's shards whole)
        same_tp = self.eng_tp is not None and not a.is_moe and bool(descs) and \
            all(int(d.get("tp_world", 1)) == self.eng_tp.world for d in descs)
        shard_mode = self.eng_tp is not None and (not any("entries" in d for d in descs) or same_tp)
        # (a TP rank pulling its shards directly needs no full-model buffer)
        flat = torch.empty(layout.total if not shard_mode else 0, dtype=dtype, device=self.device)
        w = EngineWeights(a, self.device, dtype)
        w.flat = flat
        w.tensors = layout.views(flat) if not shard_mode else {}
        if a.is_moe:
            prior = zipf_prior(a.num_experts, a.router_zipf_alpha) if a.router_zipf_alpha > 0 \
                else torch.zeros(a.num_experts)
            for i in range(a.num_layers):
                w.tensors[f"layers.{i}.mlp.router_prior"] = prior.to(self.device)
        self.weights = w
        self.shard_pull = False
        if not shard_mode:
            self.puller = ShardedWeightPuller(layout, descs, flat, a) if any("entries" in d for d in descs) \
                else WeightPuller(layout, descs, flat)
        if shard_mode:
            # whole-tensor trainer stores (data-parallel trainers): each TP rank
            # copies only its own slices, straight into its shard buffers
            from ..parallel.weight_sync import EngineShardPuller
            self.puller = EngineShardPuller(layout, descs, a, self.eng_tp.rank, self.eng_tp.world, self.device)
            ew = EngineWeights(a, self.device, dtype)
            ew.tensors = dict(self.puller.tensors)
            if a.is_moe:
                for i in range(a.num_layers):
                    ew.tensors[f"layers.{i}.mlp.router_prior"] = w.tensors[f"layers.{i}.mlp.router_prior"]
            self.shard_pull = True
            w = ew
        elif self.eng_tp is not None:
            # sharded trainer stores: every TP rank pulls the full model, then keeps
            # its own shard of the column / row-parallel tensors (persistent copies,
            # refreshed after each pull; replicated tensors stay views of the pulled buffer)
            from ..parallel.tp import shard_engine_tensors
            self.full_tensors = w.tensors
            ew = EngineWeights(a, self.device, dtype)
            ew.tensors = shard_engine_tensors(a, self.full_tensors, self.eng_tp)
            self.sharded_names = [n for n, t in ew.tensors.items() if t is not self.full_tensors.get(n)]
            self.weights_tp = ew.tensors
            w = ew
        max_len = int(rc.max_prompt_length) + int(rc.max_response_length) + 64
        # a rollout-only GPU can give the KV cache and the batch more room
        kv_gb = float(rc.get("kv_cache_gb_dedicated", 0) or rc.get("kv_cache_gb", 4.0))
        max_seqs = int(rc.get("max_num_seqs_dedicated", 0) or rc.max_num_seqs)
        self.engine = RolloutEngine(
            a, w, max_num_seqs=max_seqs, max_model_len=max_len, block_size=int(rc.block_size),
            max_num_batched_tokens=int(rc.max_num_batched_tokens), kv_cache_gb=kv_gb,
            enable_prefix_caching=bool(rc.enable_prefix_caching), use_cuda_graph=bool(rc.cuda_graph),
            keep_kv_on_update=bool(cfg.psrl.rollout_coordination.partial_rollout.get("keep_kv", False)),
            eos_token_id=None if rc.ignore_eos else self.cp.eos_id(), decode_gemm=str(cfg.rollout.get("decode_gemm", "library")),
            kv_offload_blocks=int(cfg.rollout.get("kv_offload_blocks", 0) or 0), tp=self.eng_tp)
        sm = cfg.psrl.rollout_coordination.sync_and_mig_strategy
        self.policy = SyncPolicy(sm.method, bool(cfg.psrl.rollout_coordination.partial_rollout.enable),
                                 sm.sync.get("threshold"), sm.sync.get("indicator", "request_num"))
        self._pull()
        if self.is_leader:
            self.cp.register_instance(self.instance_id, self.engine.version)
        log(f"rollout instance {self.instance_id} ready at version {self.engine.version} "
            f"({max_seqs} seqs, {kv_gb:.0f} GB KV)")

    def _pull(self) -> None:
        if self.eng_tp is not None:
            return self._tp_pull()
        t0 = time.perf_counter()
        if not self.cp.acquire_pull():
            raise TimeoutError("shared pull lock")
        copy_s = None
        try:
            v = self.cp.pull_model(self.instance_id)
            if self.device.type == "cuda":
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                nbytes = self.puller.pull()
                e1.record()
                e1.synchronize()
                copy_s = e0.elapsed_time(e1) / 1e3      # device time of the peer-load kernel
            else:
                nbytes = self.puller.pull()
        finally:
            self.cp.release_pull()
        from_v = self.engine.version
        in_flight = self.engine.num_unfinished()
        self.engine.load_weights(None, v)
        self.cp.report_pull(time.perf_counter() - t0, self.instance_id, from_v, v,
                            0 if self.engine.keep_kv_on_update else in_flight, copy_s, int(nbytes))
        self.log.record_span("PULL", time.time() - (time.perf_counter() - t0), time.perf_counter() - t0,
                             version=int(v), bytes=int(nbytes))

    def _tp_pull(self) -> None:
        """A TP instance's pull: the leader takes the shared pull lock and the
        version, every rank of the group copies the full model from the
        trainer stores and re-slices its shard, and the leader releases the
        lock once all of them are done (a gloo barrier of the group)."""
        t0 = time.perf_counter()
        box = [None]
        if self.is_leader:
            ok = bool(self.cp.acquire_pull())
            box = [(ok, self.cp.pull_model(self.instance_id) if ok else None)]
        dist.broadcast_object_list(box, src=self.eng_leader, group=self.eng_tp_cpu)
        ok, v = box[0]
        if not ok:
            raise TimeoutError("shared pull lock")
        try:
            nbytes = self.puller.pull()
            if not self.shard_pull:
                from ..parallel.tp import shard_engine_tensors
                fresh = shard_engine_tensors(self.args, self.full_tensors, self.eng_tp)
                for n in self.sharded_names:
                    self.weights_tp[n].copy_(fresh[n])
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            dist.barrier(group=self.eng_tp_cpu)
        finally:
            if self.is_leader:
                self.cp.release_pull()
        from_v = self.engine.version
        in_flight = self.engine.num_unfinished()
        self.engine.load_weights(None, v)
        if self.is_leader:
            self.cp.report_pull(time.perf_counter() - t0, self.instance_id, from_v, v,
                                0 if self.engine.keep_kv_on_update else in_flight, None, int(nbytes))

    def _coordinated_pull(self) -> None:
        """Pull granted by the control plane's coordinator; a failure quarantines
        this instance (it gets no more work) instead of ending the run."""
        try:
            self._pull()
        except Exception as exc:
            self.cp.report_sync_failure(self.instance_id, f"{type(exc).__name__}: {exc}")

    def _tp_rollout_loop(self, on_phase) -> None:
        """A TP instance: the leader reads its mailbox and the driver phase and
        broadcasts (requests, aborts, phase, pull decision) each round, so every
        rank of the group applies the same operations and steps in lockstep."""
        eng = self.engine
        leader = self.is_leader
        mb = None
        if leader:
            self.mailbox = mb = ExchangeMailbox(self.cp, self.instance_id, eng)
        seen = 0
        idle_s = 0.0
        try:
            while True:
                msg = None
                if leader:
                    reqs, aborts = mb.collect()
                    sync = bool(mb.take_sync_grant() and mb.ps_version > eng.version)
                    msg = (reqs, aborts, mb.phase, sync)
                box = [msg]
                dist.broadcast_object_list(box, src=self.eng_leader, group=self.eng_tp_cpu)
                reqs, aborts, phase, sync = box[0]
                for r in reqs:
                    eng.add_request(r)
                for rid in aborts:
                    eng.abort(rid)
                while seen < phase:
                    seen += 1
                    if leader:
                        self.cp.report_engine(self.instance_id, seen,
                                              {**{k: float(v) for k, v in eng.stats.items()}, "idle_time": idle_s})
                    on_phase(seen)
                if seen >= 2:
                    return
                if sync:
                    try:
                        self._tp_pull()
                    except Exception as exc:
                        if leader:
                            self.cp.report_sync_failure(self.instance_id, f"{type(exc).__name__}: {exc}")
                if eng.has_unfinished():
                    outs = eng.step()
                    if outs and leader:
                        mb.post(outs)
                else:
                    if leader:
                        mb.kick()
                    t_idle = time.perf_counter()
                    time.sleep(0.0005)
                    idle_s += time.perf_counter() - t_idle
        finally:
            if mb is not None:
                mb.close()
            self.mailbox = None

    def rollout_loop(self, on_phase) -> None:
        """Serve until the driver reaches the final phase; ``on_phase(p)`` runs the
        collective steps tied to phase ``p`` (same order as on the trainers)."""
        eng = self.engine
        if self.device.type == "cuda" and eng.use_cuda_graph:
            eng.capture_all()
        if self.eng_tp is not None:
            return self._tp_rollout_loop(on_phase)
        self.mailbox = mb = ExchangeMailbox(self.cp, self.instance_id, eng)
        seen = 0
        idle_s = 0.0
        # host-side fault injection for failure-detection tests: this rollout
        # rank leaves abruptly (no exception, no goodbye) after that many seconds
        exit_after = float(self.cfg.trainer.get("inject_rollout_exit_after_s", 0) or 0)
        t_enter = time.monotonic()
        try:
            while True:
                if exit_after > 0 and time.monotonic() - t_enter > exit_after:
                    os._exit(3)
                reqs, aborts = mb.collect()
                for r in reqs:
                    eng.add_request(r)
                for rid in aborts:
                    eng.abort(rid)
                while seen < mb.phase:
                    seen += 1
                    # engine counters at the start / end of the timed region
                    self.cp.report_engine(self.instance_id, seen,
                                          {**{k: float(v) for k, v in eng.stats.items()}, "idle_time": idle_s})
                    on_phase(seen)
                if seen >= 2:
                    return
                if mb.take_sync_grant() and mb.ps_version > eng.version:
                    self._coordinated_pull()
                if eng.has_unfinished():
                    outs = eng.step()
                    if outs:
                        mb.post(outs)
                else:
                    mb.kick()
                    t_idle = time.perf_counter()
                    time.sleep(0.0005)
                    idle_s += time.perf_counter() - t_idle
        finally:
            mb.close()
            self.mailbox = None

    def close(self):
        if self.rank == 0:
            with contextlib.suppress(Exception):
                self.cp.shutdown()
        self.client.close()
        if self.cp_proc is not None:
            self.cp_proc.join(timeout=30)
            if self.cp_proc.is_alive():
                self.cp_proc.terminate()


def _log_step_spans(log, step: int, t0: float, t1: float, t2: float, metrics: dict) -> None:
    """WAIT (generation wait), TRAIN and PUSH spans of one trainer step from its
    perf_counter marks; VAL / checkpoint spans from their timing metrics."""
    off = time.time() - time.perf_counter()
    log.record_span("WAIT", t0 + off, t1 - t0, step=step)
    log.record_span("TRAIN", t1 + off, t2 - t1, step=step)
    log.record_span("PUSH", t2 + off, float(metrics.get("timing_s/publish", 0.0)), step=step)
    if "timing_s/validate" in metrics:
        log.record_span("VAL", time.time() - metrics["timing_s/validate"], metrics["timing_s/validate"], step=step)


def run_disaggregated(cfg, steps: int, warmup: int, info: pdist.DistInfo | None = None):
    """Run ``warmup`` + ``steps`` training steps; returns per-rank timing dict
    (rank 0 also gets metrics, token counts and control-plane stats)."""
    info = info or pdist.init_distributed(cfg.trainer.get("device", "auto"))
    run = DisaggregatedRun(cfg, info)
    if steps is None:
        # trainer.total_training_steps counts from step 0 (a resumed run does the rest)
        steps = max(0, int(cfg.trainer.total_training_steps) - int(getattr(run, "global_step", 0)))
    is_cuda = info.device.type == "cuda"
    t_evt = {}

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
        if run.is_trainer:
            for i in range(warmup):
                m = run.trainer_step()
                if run.rank == 0:
                    log(f"warm-up step {i}: {m['timing_s/step']:.1f}s (wait {m['timing_s/gen_wait']:.1f}s), "
                        f"{m['trained_tokens']} tokens")
            if run.rank == 0:
                run.cp.set_phase(1)
            mark(1)
            for i in range(steps):
                metrics.append(run.trainer_step())
                if run.rank == 0:
                    m = metrics[-1]
                    log(f"timed step {i}: {m['timing_s/step']:.1f}s (wait {m['timing_s/gen_wait']:.1f}s), "
                        f"{m['trained_tokens']} tokens")
            if run.rank == 0:
                run.cp.set_phase(2)
            mark(2)
        else:
            try:
                run.rollout_loop(mark)
            except BaseException as exc:
                with contextlib.suppress(Exception):
                    run.cp.report_failure(run.instance_id, f"{type(exc).__name__}: {exc}")
                raise
        if is_cuda:
            torch.cuda.synchronize()
            ms = t_evt[1].elapsed_time(t_evt[2])
        else:
            ms = (t_evt["wall2"] - t_evt["wall1"]) * 1000.0
        wall = t_evt["wall2"] - t_evt["wall1"]
        # host<->device bytes of this rank inside the timed region
        xfer = [b - a for a, b in zip(t_evt["xfer1"], t_evt["xfer2"])]
        ms_max = pdist.all_reduce_max(ms, info.device)
        wall_max = pdist.all_reduce_max(wall, info.device)
        out = {"ms": ms_max, "wall_s": wall_max, "rank": run.rank, "metrics": metrics,
               "h2d": xfer[0], "d2h": xfer[1],
               "n_train": run.n_train, "world": run.world}
        if run.rank == 0:
            out["tokens"] = sum(int(m["trained_tokens"]) for m in metrics)
            st = run.cp.stats()
            out["sync"] = st["sync"]
            out["manager"] = st["manager"]
            out["cp"] = st
        pdist.barrier()
    finally:
        run.close()
    return out


def run_disaggregated_bench(args, placement: str = "disaggregated"):
    """bench.py entry for torch.distributed.run launches (N >= 1 ranks):
    ``placement`` is ``disaggregated`` (trainer ranks + rollout ranks) or
    ``hybrid`` (every rank trains and serves rollout, :mod:`.hybrid`)."""
    from ..bench.rl_bench import build_cfg
    from ..ops import _ext
    from ..utils.clocks import ClockSampler

    info = pdist.init_distributed("cuda", timeout_s=900)
    cfg = build_cfg(args, info.world_size)
    sampler = ClockSampler(list(range(info.world_size))).start() if info.rank == 0 else None
    l0 = _ext.launches()
    if placement == "hybrid":
        from .hybrid import run_hybrid
        res = run_hybrid(cfg, args.steps, args.warmup, info)
        n_train = res["world"]
        par = f"hybrid: train dp{n_train} + {n_train} overlapped rollout instances (tp1), local weight sync"
    else:
        res = run_disaggregated(cfg, args.steps, args.warmup, info)
        n_train = res["n_train"]
        ac = cfg.actor
        mp = [f"{k}{int(ac.get(key, 1) or 1)}" for k, key in (("tp", "tensor_parallel_size"),
                                                               ("cp", "context_parallel_size"),
                                                               ("pp", "pipeline_parallel_size"),
                                                               ("ep", "expert_parallel_size"))
              if int(ac.get(key, 1) or 1) > 1]
        g = 1
        for m in mp:
            g *= int(m[2:]) if not m.startswith("ep") else 1
        train = f"dp{n_train // g} (sharded)" + ("".join(" x " + m for m in mp))
        par = f"train {train} + rollout dp{res['world'] - n_train} (tp1), NVLink weight pull"
    launches = pdist.all_reduce_sum(float(_ext.launches() - l0), info.device)
    # bytes copied host<->device inside the timed region, all ranks
    h2d = pdist.all_reduce_sum(float(res["h2d"]), info.device)
    d2h = pdist.all_reduce_sum(float(res["d2h"]), info.device)
    clocks = sampler.stop() if sampler else None
    pdist.destroy()
    if info.rank != 0:
        return None
    res.update({
        "launches": launches, "clocks": clocks,
        "h2d": h2d / max(1, args.steps), "d2h": d2h / max(1, args.steps),
        "prompts_per_step": cfg.psrl.staleness_buffer_entries,
        "trajectories_per_step": cfg.psrl.staleness_buffer_entries * cfg.psrl.rollout_n,
        "parallelism": par,
        "api": "HybridRun.step" if placement == "hybrid" else "DisaggregatedRun.trainer_step",
    })
    return res
