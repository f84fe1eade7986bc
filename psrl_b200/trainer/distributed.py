"""Disaggregated asynchronous RL over N processes (one per device).

Ranks ``[0, T)`` train (sharded data parallel over an NCCL group), ranks
``[T, N)`` each run one rollout instance.  Rank 0 additionally hosts the
Parameter Server, the dispatcher (agent-loop manager, reward) and an RPC
service the rollout ranks talk to (this replaces the reference's Ray actors,
the SMG router's gRPC admission calls and the TransferQueue hop: trajectories
travel back in the same RPC that fetches new work).

Weights: every trainer rank publishes its parameters into its
:class:`~psrl_b200.parallel.weight_sync.WeightStore` (HBM) under the PS
exclusive-push lock; rollout ranks pull slices from all trainers over NVLink
under the shared-pull lock whenever their sync policy allows.

On CPU the same code runs with gloo and a shared-memory store (the
world_size=2 plumbing configuration).
"""

from __future__ import annotations

import os
import sys
import threading
import time

import torch
import torch.distributed as dist

from ..agent.data import DataProcessor
from ..agent.manager import AgentLoopManager
from ..config import redundant_settings
from ..models import build_model, model_args_from_config
from ..models.qwen import zipf_prior
from ..parallel import dist as pdist
from ..parallel.weight_sync import WeightLayout, WeightPuller, WeightStore
from ..ps import PSManager
from ..reward import RewardManager
from ..rollout.engine import EngineWeights, RolloutEngine
from ..rollout.instance import SyncPolicy
from ..utils.rpc import RPCClient, RPCServer
from .actor import PolicyWorker
from .driver import compute_batch_advantages


class DispatcherService:
    """Rank-0 control plane exposed to rollout ranks."""

    def __init__(self, cfg, ps: PSManager, manager: AgentLoopManager, n_train: int):
        self.cfg = cfg
        self.ps = ps
        self.manager = manager
        self.n_train = n_train
        self.stores: dict[int, dict] = {}
        self.layout = None
        self.phase = 0
        self._cv = threading.Condition()
        self.sync_stats = {"pulls": 0, "pull_s": 0.0}
        self.last_seen: dict = {}
        self.failed: dict = {}

    # setup
    def register_store(self, trainer_rank: int, desc: dict) -> None:
        with self._cv:
            self.stores[trainer_rank] = desc
            self._cv.notify_all()

    def set_layout(self, layout) -> None:
        with self._cv:
            self.layout = layout
            self._cv.notify_all()

    def get_stores(self, timeout: float = 600.0) -> tuple:
        with self._cv:
            ok = self._cv.wait_for(lambda: len(self.stores) == self.n_train and self.layout is not None, timeout)
            if not ok:
                raise TimeoutError("trainer stores were not registered in time")
            return self.layout, [self.stores[r] for r in range(self.n_train)]

    def register_instance(self, instance_id, version: int) -> None:
        self.ps.register_rollout_instance(tuple(instance_id), version)

    # steady state
    def report_failure(self, instance_id, message: str) -> None:
        self.failed[tuple(instance_id)] = message

    def exchange(self, instance_id, version: int, free_slots: int, outputs: list):
        instance_id = tuple(instance_id)
        self.last_seen[instance_id] = time.monotonic()
        if outputs:
            self.manager.on_complete(outputs, instance_id)
        reqs = self.manager.take_work(instance_id, version, free_slots) if free_slots > 0 else []
        aborts = self.manager.take_aborts(instance_id)
        return reqs, aborts, self.ps.get_ps_model_version(), self.phase

    def acquire_pull(self, timeout: float = 600.0) -> bool:
        return self.ps.acquire_shared_pull(timeout)

    def release_pull(self) -> None:
        self.ps.release_shared_pull()

    def pull_model(self, instance_id) -> int:
        v, _ = self.ps.pull_model(tuple(instance_id))
        return v

    def report_pull(self, seconds: float) -> None:
        self.sync_stats["pulls"] += 1
        self.sync_stats["pull_s"] += seconds

    def set_phase(self, p: int) -> None:
        self.phase = p


def log(msg: str) -> None:
    r = os.environ.get("RANK", "0")
    print(f"[rank {r} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def _role_split(world: int, cfg) -> int:
    t = int(cfg.psrl.deployment.get("train_ngpus", 0) or 0)
    if t <= 0 or t >= world:
        t = max(1, world // 2)
    return t


def _broadcast_objs(obj, src: int, group) -> object:
    box = [obj]
    dist.broadcast_object_list(box, src=src, group=group)
    return box[0]


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
        if self.is_trainer and self.n_train > 1:
            # created by the trainer ranks only (group-local synchronisation)
            self.train_group = pdist.new_subgroup(trainer_ranks, backend=backend)
            self.train_cpu_group = pdist.new_subgroup(trainer_ranks, backend="gloo")
        self.args = model_args_from_config(cfg.model)
        self.port = int(os.environ.get("MASTER_PORT", "29511")) + 17
        self.trained_tokens = 0
        self.global_step = 0
        self.server = None
        self.liveness_s = float(cfg.trainer.get("liveness_timeout_s", 300))
        self.buffer_timeout_s = float(cfg.trainer.get("buffer_timeout_s", 1800))
        log(f"role split: {self.n_train} trainer rank(s), {self.world - self.n_train} rollout rank(s)")
        if self.rank == 0:
            rn, _, _, _ = redundant_settings(cfg)
            self.ps = PSManager.from_config(cfg)
            self.data = DataProcessor(cfg, self.args.vocab_size, rn)
            self.reward = RewardManager(cfg, self.data.tokenizer)
            self.manager = AgentLoopManager(cfg, self.ps, self.data, self.reward)
            self.svc = DispatcherService(cfg, self.ps, self.manager, self.n_train)
            self.server = RPCServer({"svc": self.svc}, port=self.port)
        pdist.barrier()
        log("control plane up")
        self.client = None if self.rank == 0 else RPCClient(("127.0.0.1", self.port))
        self.svc_proxy = self.svc if self.rank == 0 else self.client.proxy("svc")
        if self.is_trainer:
            self._init_trainer()
        else:
            self._init_rollout()

    # ------------------------------------------------------------ trainer
    def _init_trainer(self):
        cfg = self.cfg
        self.actor = PolicyWorker(cfg, self.args, self.device, dp_group=self.train_group,
                                  seed=int(cfg.trainer.seed), dp_rank=self.rank, dp_world=self.n_train)
        self.layout = WeightLayout.from_dp(self.actor.dp)
        mode = "hbm" if (cfg.psrl.ps_mode == "hbm" and self.device.type == "cuda") else "cpu"
        self.store = WeightStore(self.layout, self.device, mode)
        self.store.publish(self.actor.dp.flat, 0)
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        if self.rank == 0:
            self.svc.set_layout(self.layout)
        self.svc_proxy.register_store(self.rank, self.store.descriptor())
        log(f"trainer ready: {self.layout.nbytes / 2**30:.2f} GiB published store ({mode})")

    def trainer_step(self) -> dict:
        b = self.global_step
        t0 = time.perf_counter()
        trajs = None
        if self.rank == 0:
            t_wait = time.monotonic()
            while not self.manager.buffer_ready(b):
                if self.svc.failed:
                    raise RuntimeError(f"rollout instance failed: {self.svc.failed}")
                now = time.monotonic()
                stale = [i for i, t in self.svc.last_seen.items() if now - t > self.liveness_s]
                if stale or now - t_wait > self.buffer_timeout_s:
                    raise TimeoutError(f"buffer {b} not ready: silent instances {stale}, "
                                       f"{self.manager.snapshot()}")
                time.sleep(0.002)
            trajs = self.manager.consume(b)
            for t in trajs:
                t.old_logprobs = t.rollout_logprobs
            adv_metrics = compute_batch_advantages(self.cfg, trajs)
        t1 = time.perf_counter()
        if self.n_train > 1:
            trajs = _broadcast_objs(trajs, 0, self.train_cpu_group)
        metrics = self.actor.update_policy(trajs, float(self.cfg.rollout.temperature))
        t2 = time.perf_counter()
        # publish: PS exclusive lock (rank 0) -> every trainer writes its store -> version bump
        if self.rank == 0:
            if not self.ps.acquire_exclusive_push(timeout=600):
                raise TimeoutError("exclusive push lock")
        if self.n_train > 1:
            dist.barrier(group=self.train_cpu_group)
        self.store.publish(self.actor.dp.flat, b + 1)
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        if self.n_train > 1:
            dist.barrier(group=self.train_cpu_group)
        if self.rank == 0:
            self.ps.push_model(b + 1)
            self.ps.release_exclusive_push()
            metrics.update(adv_metrics)
        self.global_step += 1
        ntok = sum(len(t.prompt_ids) + t.response_len for t in trajs)
        self.trained_tokens += ntok
        metrics.update({"step": b, "trained_tokens": ntok, "num_trajectories": len(trajs),
                        "timing_s/gen_wait": t1 - t0, "timing_s/train": t2 - t1,
                        "timing_s/step": time.perf_counter() - t0})
        return metrics

    # ------------------------------------------------------------ rollout
    def _init_rollout(self):
        cfg, a = self.cfg, self.args
        rc = cfg.rollout
        self.instance_id = (self.rank - self.n_train, 0)
        log("rollout: waiting for trainer stores")
        layout, descs = self.svc_proxy.get_stores()
        self.layout = layout
        dtype = layout.dtype
        flat = torch.empty(layout.total, dtype=dtype, device=self.device)
        w = EngineWeights(a, self.device, dtype)
        w.flat = flat
        w.tensors = layout.views(flat)
        if a.is_moe:
            prior = zipf_prior(a.num_experts, a.router_zipf_alpha) if a.router_zipf_alpha > 0 \
                else torch.zeros(a.num_experts)
            for i in range(a.num_layers):
                w.tensors[f"layers.{i}.mlp.router_prior"] = prior.to(self.device)
        self.weights = w
        self.puller = WeightPuller(layout, descs, flat)
        max_len = int(rc.max_prompt_length) + int(rc.max_response_length) + 64
        self.engine = RolloutEngine(
            a, w, max_num_seqs=int(rc.max_num_seqs), max_model_len=max_len, block_size=int(rc.block_size),
            max_num_batched_tokens=int(rc.max_num_batched_tokens), kv_cache_gb=float(rc.get("kv_cache_gb", 4.0)),
            enable_prefix_caching=bool(rc.enable_prefix_caching), use_cuda_graph=bool(rc.cuda_graph),
            keep_kv_on_update=bool(cfg.psrl.rollout_coordination.partial_rollout.get("keep_kv", False)),
            eos_token_id=None if rc.ignore_eos else 2)
        sm = cfg.psrl.rollout_coordination.sync_and_mig_strategy
        self.policy = SyncPolicy(sm.method, bool(cfg.psrl.rollout_coordination.partial_rollout.enable),
                                 sm.sync.get("threshold"), sm.sync.get("indicator", "request_num"))
        self._pull()
        self.svc_proxy.register_instance(self.instance_id, self.engine.version)
        log(f"rollout instance {self.instance_id} ready at version {self.engine.version}")

    def _pull(self) -> None:
        t0 = time.perf_counter()
        if not self.svc_proxy.acquire_pull():
            raise TimeoutError("shared pull lock")
        try:
            v = self.svc_proxy.pull_model(self.instance_id)
            self.puller.pull()
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
        finally:
            self.svc_proxy.release_pull()
        self.engine.load_weights(None, v)
        self.svc_proxy.report_pull(time.perf_counter() - t0)

    def rollout_loop(self, on_phase) -> None:
        """Serve until the driver reaches the final phase; ``on_phase(p)`` runs the
        collective steps tied to phase ``p`` (same order as on the trainers)."""
        eng = self.engine
        seen = 0
        last = 0.0
        ps_v = eng.version
        pending: list = []
        while True:
            if eng.has_unfinished():
                pending.extend(eng.step())
            free = eng.max_num_seqs - eng.num_unfinished()
            now = time.monotonic()
            if pending or (free >= 16 and now - last > 0.002) or now - last > 0.02:
                reqs, aborts, ps_v, phase = self.svc_proxy.exchange(self.instance_id, eng.version, free, pending)
                pending = []
                last = now
                for rid in aborts:
                    o = eng.abort(rid)
                    del o
                for r in reqs:
                    eng.add_request(r)
                while seen < phase:
                    seen += 1
                    on_phase(seen)
                if seen >= 2:
                    return
            if self.policy.should_sync(eng, ps_v):
                self._pull()
            if not eng.has_unfinished():
                time.sleep(0.001)

    def close(self):
        if self.client is not None:
            self.client.close()
        if self.server is not None:
            self.server.close()


def run_disaggregated(cfg, steps: int, warmup: int, info: pdist.DistInfo | None = None):
    """Run ``warmup`` + ``steps`` training steps; returns per-rank timing dict
    (rank 0 also gets metrics and token counts)."""
    info = info or pdist.init_distributed(cfg.trainer.get("device", "auto"))
    run = DisaggregatedRun(cfg, info)
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

    metrics = []
    if run.is_trainer:
        for i in range(warmup):
            m = run.trainer_step()
            if run.rank == 0:
                log(f"warm-up step {i}: {m['timing_s/step']:.1f}s, {m['trained_tokens']} tokens")
        if run.rank == 0:
            run.svc.set_phase(1)
        mark(1)
        for i in range(steps):
            metrics.append(run.trainer_step())
            if run.rank == 0:
                log(f"timed step {i}: {metrics[-1]['timing_s/step']:.1f}s")
        if run.rank == 0:
            run.svc.set_phase(2)
        mark(2)
    else:
        try:
            run.rollout_loop(mark)
        except BaseException as exc:
            try:
                run.svc_proxy.report_failure(run.instance_id, f"{type(exc).__name__}: {exc}")
            except Exception:
                pass
            raise
    if is_cuda:
        torch.cuda.synchronize()
        ms = t_evt[1].elapsed_time(t_evt[2])
    else:
        ms = (t_evt["wall2"] - t_evt["wall1"]) * 1000.0
    wall = t_evt["wall2"] - t_evt["wall1"]
    ms_max = pdist.all_reduce_max(ms, info.device)
    wall_max = pdist.all_reduce_max(wall, info.device)
    out = {"ms": ms_max, "wall_s": wall_max, "rank": run.rank, "metrics": metrics,
           "n_train": run.n_train, "world": run.world}
    if run.rank == 0:
        out["tokens"] = sum(m["trained_tokens"] for m in metrics)
        out["sync"] = dict(run.svc.sync_stats)
        out["manager"] = run.manager.snapshot()
    pdist.barrier()
    run.close()
    return out


def run_disaggregated_bench(args, placement: str = "disaggregated"):
    """bench.py entry for torch.distributed.run launches (N >= 1 ranks):
    ``placement`` is ``disaggregated`` (trainer ranks + rollout ranks) or
    ``hybrid`` (every rank trains and serves rollout, :mod:`.hybrid`)."""
    from bench import build_cfg
    from ..ops import _ext
    from ..utils import transfer
    from ..utils.clocks import ClockSampler

    info = pdist.init_distributed("cuda", timeout_s=900)
    cfg = build_cfg(args, info.world_size)
    sampler = ClockSampler(list(range(info.world_size))).start() if info.rank == 0 else None
    l0 = _ext.launches()
    b0, o0 = transfer.snapshot()
    if placement == "hybrid":
        from .hybrid import run_hybrid
        res = run_hybrid(cfg, args.steps, args.warmup, info)
        n_train = res["world"]
        par = f"hybrid: train dp{n_train} + {n_train} overlapped rollout instances (tp1), local weight sync"
    else:
        res = run_disaggregated(cfg, args.steps, args.warmup, info)
        n_train = res["n_train"]
        par = f"train dp{n_train} + rollout dp{res['world'] - n_train} (tp1)"
    launches = pdist.all_reduce_sum(float(_ext.launches() - l0), info.device)
    b1, o1 = transfer.snapshot()
    h2d = pdist.all_reduce_sum(float(b1 - b0), info.device)
    d2h = pdist.all_reduce_sum(float(o1 - o0), info.device)
    clocks = sampler.stop() if sampler else None
    pdist.destroy()
    if info.rank != 0:
        return None
    res.update({
        "launches": launches, "clocks": clocks,
        "h2d": h2d / max(1, args.steps + args.warmup), "d2h": d2h / max(1, args.steps + args.warmup),
        "global_batch": cfg.psrl.staleness_buffer_entries * cfg.psrl.rollout_n,
        "parallelism": par,
    })
    return res
