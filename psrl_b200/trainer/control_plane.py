"""The control plane as its own CPU process, and the GPU ranks' clients of it.

:class:`ControlPlane` hosts the Parameter Server (C8: versions, staleness
inventory, request tracker, push/pull lock), the agent-loop manager (C12:
dispatch-ahead bound, admission = Reserve, reward, Occupy, staleness aborts)
and a batch server.  It runs in one CPU-only process spawned by rank 0
(:func:`spawn_control_plane`), so its Python work never competes for the GIL of
a process that drives a GPU; every GPU rank reaches it over the RPC transport
(:mod:`psrl_b200.utils.rpc`).  This takes the place of the reference's Ray
actors for the PS and the agent-loop manager, of the router's admission calls
and of the TransferQueue hop (``psrl/ps/ps_manager.py``,
``psrl/workers/agent_loop/manager.py``, ``psrl/trainer/ppo/ray_trainer.py``).

* Rollout instances call ``exchange`` (finished trajectories in; new requests,
  aborts, the PS version and the run phase out) from an
  :class:`ExchangeMailbox` thread, so an engine never waits on the control
  plane between decode steps.
* Trainer ranks call ``get_batch(b, rank)``: the first caller waits until
  staleness buffer ``b`` is READY (failing fast when an instance reported an
  error or went silent), consumes it, computes advantages and plans the PPO
  mini-batches with a token-balanced split over the data-parallel ranks; each
  rank receives only its own trajectories plus its plan, so no rank unpickles
  the whole batch.
* After every trainer rank finished its optimizer step, rank 0 calls
  ``push_model(v)`` (PS version bump under the exclusive push lock).
"""

from __future__ import annotations

import threading
import time

from ..utils.rpc import RPCClient, RPCServer


class ControlPlane:
    def __init__(self, cfg, vocab_size: int, n_train: int, liveness_s: float = 300.0):
        from ..agent.data import DataProcessor
        from ..agent.manager import AgentLoopManager
        from ..config import redundant_settings
        from ..ps import PSManager
        from ..reward import RewardManager
        self.cfg = cfg
        rn, _, _, _ = redundant_settings(cfg)
        self.ps = PSManager.from_config(cfg)
        self.data = DataProcessor(cfg, vocab_size, rn)
        self.reward = RewardManager(cfg, self.data.tokenizer)
        self.manager = AgentLoopManager(cfg, self.ps, self.data, self.reward)
        self.n_train = int(n_train)
        self.liveness_s = float(liveness_s)
        self.phase = 0
        self.last_seen: dict = {}
        self.failed: dict = {}
        self.sync_stats = {"pulls": 0, "pull_s": 0.0, "copies": 0, "copy_s": 0.0, "bytes": 0}
        self.exchange_stats = {"calls": 0, "outputs": 0, "requests": 0}
        self.stores: dict[int, dict] = {}
        self.layout = None
        # rollout coordination (C16): weight-sync gating and load-balanced
        # migration over the instances' reported states
        from ..rollout.coordinator import CoordinatorConfig, RolloutCoordinator
        self.coord = RolloutCoordinator(CoordinatorConfig.from_cfg(cfg), self.ps.get_ps_model_version)
        from ..rollout.router import Router
        self.router = Router.from_cfg(cfg)
        self.states: dict = {}
        sm = cfg.psrl.rollout_coordination.sync_and_mig_strategy
        self.coord_interval_s = float(sm.get("check_interval_in_ms", 100)) / 1000.0
        self._last_mig = 0.0
        self._granted: dict = {}
        self.engine_stats: dict = {}     # instance -> phase -> engine counters
        self.mig_stats = {"rounds": 0, "requests": 0}
        self._cv = threading.Condition()
        self._batches: dict[int, dict] = {}
        self._batch_locks: dict[int, threading.Lock] = {}
        self._pre: dict[int, dict] = {}     # buffer -> request id -> per-sample fields computed early
        self._done = threading.Event()
        # validation (trainer.test_freq): requests handed to instances before
        # training work, their completions kept out of the training buffers
        self._val_queue: list = []
        self._val_pending: dict = {}         # request id -> (prompt item, meta)
        self._val_done: list = []
        self._val_round = 0
        # resume (trainer.resume_mode): data cursor and PS version of the latest
        # checkpoint, set before any instance takes work
        # engine statistics as JSON lines (trainer.engine_stats_path), at most one
        # snapshot per instance per trainer.engine_stats_interval_s
        self._stats_rec = None
        if cfg.trainer.get("engine_stats_path", None):
            from ..rollout.stats import StatsRecorder
            self._stats_rec = StatsRecorder(str(cfg.trainer.engine_stats_path))
        self._stats_every = float(cfg.trainer.get("engine_stats_interval_s", 1.0) or 1.0)
        self._stats_last: dict = {}
        self._resumed = None
        if str(cfg.trainer.get("resume_mode", "disable")) != "disable":
            import torch as _torch
            from ..utils.checkpoint import find_latest, step_dir
            root = cfg.trainer.get("resume_from_path") or cfg.trainer.default_local_dir
            step = find_latest(root)
            if step is not None:
                import os as _os
                meta = _torch.load(_os.path.join(step_dir(root, step), "data.pt"), weights_only=False)
                if meta.get("data"):
                    self.data.load_state_dict(meta["data"])
                self.ps.init_model_version_for_resume(step + 1)
                self.manager.initial_ps_version = step
                self.manager.request_counter = 0
                self._resumed = int(step)

    # ----------------------------------------------------------------- setup
    def ping(self) -> bool:
        return True

    def eos_id(self):
        return self.data.tokenizer.eos_id

    def register_store(self, trainer_rank: int, desc: dict) -> None:
        with self._cv:
            self.stores[int(trainer_rank)] = desc
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
        iid = tuple(instance_id)
        self.ps.register_rollout_instance(iid, int(version))
        self.last_seen[iid] = time.monotonic()

    def report_sync_failure(self, instance_id, message: str) -> None:
        """A weight pull failed on an instance: quarantine it (no more requests);
        the rest of the run continues on the healthy instances."""
        from ..rollout.router import InstanceState
        iid = tuple(instance_id)
        s = self.states.setdefault(iid, InstanceState(iid))
        self.coord.syncing.discard(iid)
        self.coord.quarantine(s)
        self.sync_stats.setdefault("failures", []).append(f"{iid}: {message}")

    def report_failure(self, instance_id, message: str) -> None:
        self.failed[tuple(instance_id)] = message

    def set_phase(self, p: int) -> None:
        self.phase = int(p)

    def shutdown(self) -> None:
        self.manager.flush_turn_records()
        self._done.set()

    # --------------------------------------------------------------- rollout
    def exchange(self, instance_id, version: int, free_slots: int, outputs: list, state: dict | None = None):
        """One round trip of a rollout instance: finished trajectories in; new
        requests, aborts (staleness aborts and migration moves), the PS version,
        the run phase and the coordinator's sync decision out."""
        iid = tuple(instance_id)
        now = time.monotonic()
        self.last_seen[iid] = now
        if outputs and any(o.request_id >= self.VAL_RID_BASE for o in outputs):
            # validation samples (late ones, after a timed-out round, are dropped)
            with self._cv:
                for o in outputs:
                    item = self._val_pending.pop(o.request_id, None) if o.request_id >= self.VAL_RID_BASE else None
                    if item is not None:
                        self._val_done.append((item, o))
                self._cv.notify_all()
            outputs = [o for o in outputs if o.request_id < self.VAL_RID_BASE]
        if outputs:
            self.manager.on_complete(outputs, iid)
        sync = self._coordinate(iid, int(version), state, now)
        if self._stats_rec is not None and state and now - self._stats_last.get(iid, -1e9) >= self._stats_every:
            self._stats_last[iid] = now
            self._stats_rec.record({"instance_id": list(iid), "version": int(version), "ts": time.time(),
                                    "num_running": int(state.get("running", 0)),
                                    "num_waiting": int(state.get("waiting", 0)),
                                    "kv_usage": float(state.get("kv_usage", 0.0)),
                                    "gen_throughput": float(state.get("throughput", 0.0))})
        quarantined = iid in self.coord.quarantined
        reqs = []
        if free_slots > 0 and not quarantined and self._val_queue:
            with self._cv:
                reqs, self._val_queue = self._val_queue[:free_slots], self._val_queue[free_slots:]
            free_slots -= len(reqs)
        if free_slots > 0 and not quarantined:
            me = self.states[iid]
            peers = [s for i, s in self.states.items() if i not in self.coord.quarantined]
            accept = None
            if len(peers) > 1:
                # routing policy in pull mode (request balance, stickiness, cache affinity, ...)
                accept = lambda req: self.router.accepts(req, me, peers)          # noqa: E731
            work = self.manager.take_work(iid, int(version), int(free_slots), accept)
            for r in work:
                self.router.assigned(r, me)
            reqs = reqs + work
        aborts = self.manager.take_aborts(iid)
        st = self.exchange_stats
        st["calls"] += 1
        st["outputs"] += len(outputs)
        st["requests"] += len(reqs)
        return reqs, aborts, self.ps.get_ps_model_version(), self.phase, sync

    def _coordinate(self, iid, version: int, state: dict | None, now: float) -> bool:
        """Update the instance's state; decide whether it syncs now and, every
        check interval, plan a migration round between instances."""
        from ..rollout.router import InstanceState
        s = self.states.get(iid)
        if s is None:
            s = self.states[iid] = InstanceState(iid)
        s.version = version
        if state:
            s.num_running = int(state.get("running", 0))
            s.num_waiting = int(state.get("waiting", 0))
            s.kv_usage = float(state.get("kv_usage", 0.0))
            s.throughput = float(state.get("throughput", 0.0))
        if iid in self.coord.syncing and (version >= self.ps.get_ps_model_version()
                                          or now - self._granted.get(iid, now) > 60.0):
            self.coord.syncing.discard(iid)        # the instance reports the new version (or the grant lapsed)
            s.paused = False
        sync = self.coord.should_sync(s)
        if sync:
            self.coord.syncing.add(iid)
            self._granted[iid] = now
            s.paused = True
        if self.coord.cfg.mig_enable and now - self._last_mig >= self.coord_interval_s:
            self._last_mig = now
            for src, dst, n in self.coord.plan_migration(list(self.states.values())):
                moved = self.manager.migrate(src, dst, n)
                if moved:
                    self.mig_stats["rounds"] += 1
                    self.mig_stats["requests"] += moved
        return sync

    VAL_RID_BASE = 1 << 50

    def resumed_step(self):
        """The checkpoint step this run resumed from (None: a fresh start)."""
        return self._resumed

    def checkpoint_meta(self) -> dict:
        """What a checkpoint keeps of the control plane: the data cursor and the PS version."""
        return {"data": self.data.state_dict(), "ps_version": self.ps.get_ps_model_version()}

    def validate(self, num_prompts: int | None = None, timeout_s: float = 1800.0) -> dict:
        """Generate on the validation prompts on the rollout instances and score
        them (``val/score_mean``, ``val/response_length/mean``,
        ``val/num_samples``).  The requests go out before any training work in
        the instances' next exchanges and carry the current PS version; their
        completions never reach the training buffers.  Sampling as in the
        one-process trainer's validation: ``trainer.val_temperature`` (0 =
        greedy), ``psrl.val_rollout_n`` samples per prompt (the reference's
        ``test_freq`` validation, ``psrl/trainer/ppo/ray_trainer.py``)."""
        from ..rollout.engine import GenRequest, SamplingParams
        from .batch import Trajectory
        cfg = self.cfg
        n = int(num_prompts if num_prompts is not None else cfg.data.get("val_size", 32))
        per = max(1, int(cfg.psrl.get("val_rollout_n", 1)))
        temp = float(cfg.trainer.get("val_temperature", 0.0))
        rc = cfg.rollout
        v = self.ps.get_ps_model_version()
        items = self.data.validation_items(n)
        with self._cv:
            self._val_round += 1
            base = self.VAL_RID_BASE + self._val_round * (1 << 32)
            for i, it in enumerate(items):
                for j in range(per):
                    rid = base + i * per + j
                    mt = int(it.response_lens[j % len(it.response_lens)]) if it.response_lens \
                        else int(rc.max_response_length)
                    params = SamplingParams(temperature=temp, top_p=1.0, top_k=-1, max_tokens=mt,
                                            ignore_eos=bool(rc.ignore_eos), seed=rid)
                    meta = dict(it.meta)
                    if it.answer is not None:
                        meta["answer"] = it.answer
                    self._val_queue.append(GenRequest(rid, list(it.prompt_ids), params, v, meta))
                    self._val_pending[rid] = (it, meta)
            ok = self._cv.wait_for(lambda: not self._val_pending, timeout_s)
            done, self._val_done = self._val_done, []
            if not ok:
                self._val_queue.clear()
                self._val_pending.clear()
                raise TimeoutError(f"validation: {len(done)} of {n * per} samples in {timeout_s:.0f} s")
        scores, lens = [], []
        for (it, meta), o in done:
            tr = Trajectory(uid=it.uid, request_id=o.request_id, prompt_ids=list(o.prompt_ids),
                            response_ids=list(o.output_ids), rollout_logprobs=list(o.logprobs), meta=meta)
            scores.append(float(self.reward.score(tr)["score"]))
            lens.append(len(o.output_ids))
        m = len(scores)
        return {"val/score_mean": sum(scores) / max(1, m), "val/response_length/mean": sum(lens) / max(1, m),
                "val/num_samples": m}

    def acquire_pull(self, timeout: float = 600.0) -> bool:
        return self.ps.acquire_shared_pull(timeout)

    def release_pull(self) -> None:
        self.ps.release_shared_pull()

    def pull_model(self, instance_id, seconds: float | None = None) -> int:
        v, _ = self.ps.pull_model(tuple(instance_id))
        if seconds is not None:
            self.report_pull(seconds)
        return v

    def report_engine(self, instance_id, phase: int, stats: dict) -> None:
        """Engine counters of a rollout instance at a phase boundary of the run."""
        self.engine_stats.setdefault(tuple(instance_id), {})[int(phase)] = dict(stats)

    def rollout_summary(self) -> dict | None:
        """Rollout engines over the timed region (between phase 1 and 2 reports),
        summed over instances: generated tokens, decode / prefill time and rate,
        idle time, preemptions."""
        keys = ("decode_tokens", "decode_steps", "decode_time", "prefill_tokens", "prefill_time", "idle_time",
                "preemptions", "cached_tokens")
        tot = {k: 0.0 for k in keys}
        n = 0
        for per in self.engine_stats.values():
            if 1 in per and 2 in per:
                n += 1
                for k in keys:
                    tot[k] += per[2].get(k, 0.0) - per[1].get(k, 0.0)
        if not n:
            return None
        out = {"instances": n, **{k: round(v, 3) for k, v in tot.items()}}
        out["decode_tok_per_s_per_instance"] = round(tot["decode_tokens"] / max(tot["decode_time"], 1e-9), 1)
        out["prefill_tok_per_s_per_instance"] = round(tot["prefill_tokens"] / max(tot["prefill_time"], 1e-9), 1)
        return out

    def report_pull(self, seconds: float, instance_id=None, from_version: int = -1, to_version: int = -1,
                    interrupted: int = 0, copy_seconds: float | None = None, nbytes: int = 0) -> None:
        """One weight pull of a rollout instance: wall time (lock, version RPC,
        copy, engine swap) and, when known, the device time of the copy kernel
        and the bytes it moved."""
        self.sync_stats["pulls"] += 1
        self.sync_stats["pull_s"] += float(seconds)
        if copy_seconds is not None:
            self.sync_stats["copies"] += 1
            self.sync_stats["copy_s"] += float(copy_seconds)
            self.sync_stats["bytes"] = int(nbytes)
        if instance_id is not None:
            from ..rollout.coordinator import SyncRecord
            self.coord.history.append(SyncRecord(tuple(instance_id), int(from_version), int(to_version),
                                                 float(seconds), int(interrupted), True))

    # --------------------------------------------------------------- trainer
    def _wait_ready(self, b: int, timeout_s: float) -> None:
        t0 = time.monotonic()
        t_act = t0
        while not self.manager.buffer_ready(b):
            if self.failed:
                raise RuntimeError(f"rollout instance failed: {self.failed}")
            now = time.monotonic()
            if now - t_act > self.manager.filter_patience_s:
                t_act = now
                self.manager.handle_waiting_buffer(b)
            silent = [i for i, t in self.last_seen.items() if now - t > self.liveness_s]
            if silent or now - t0 > timeout_s:
                raise TimeoutError(f"buffer {b} not ready: silent instances {silent}, {self.manager.snapshot()}")
            time.sleep(0.002)

    # ------------------------------------------- fine-grain overlap (recompute)
    def progress(self, b: int) -> tuple:
        """(committed entries at the head of buffer ``b``, buffer READY,
        entries that make it READY)."""
        b = int(b)
        return self.manager.occupied_prefix(b), self.manager.buffer_ready(b), int(self.manager.ready_entries)

    def peek_chunk(self, b: int, lo: int, hi: int) -> list:
        """Trajectories of entries [lo, hi) of buffer ``b`` (not consumed), for
        per-sample stages that run while the buffer fills."""
        return self.manager.peek(int(b), int(lo), int(hi))

    def post_per_sample(self, b: int, fields: dict) -> None:
        """Per-sample results (``{request_id: {field: list}}``: old / ref
        log-probs, values) computed on trainer ranks before the buffer was
        consumed; :meth:`_build` attaches them to the trajectories."""
        with self._cv:
            if int(b) in self._batches:
                return          # already built: the step computes what is missing
            self._pre.setdefault(int(b), {}).update(fields)

    def _build(self, b: int, dp_world: int, timeout_s: float) -> dict:
        from ..trainer.actor import plan_update
        from ..trainer.driver import compute_batch_advantages
        self._wait_ready(b, timeout_s)
        trajs = self.manager.consume(b)
        use_rollout_lp = bool(self.cfg.psrl.log_prob.enable_rollout_engine_log_prob)
        with self._cv:
            pre = self._pre.pop(int(b), {})
        for t in trajs:
            t.old_logprobs = t.rollout_logprobs if use_rollout_lp else None
            for k, v in pre.get(t.request_id, {}).items():
                setattr(t, k, v)
        if self.cfg.critic.enable:
            # GAE needs the critic's values: the trainer ranks compute advantages on
            # their own shares (whitened with global statistics)
            sc = [t.reward for t in trajs]
            adv_metrics = {"critic/score_mean": sum(sc) / max(1, len(sc)), "critic/score_max": max(sc, default=0.0),
                           "critic/score_min": min(sc, default=0.0)}
        else:
            adv_metrics = compute_batch_advantages(self.cfg, trajs)
        plans = plan_update(trajs, int(self.cfg.actor.ppo_mini_batch_size), dp_world)
        per_rank = {}
        for r in range(dp_world):
            need = sorted({i for mine, _, _ in plans[r] for i in mine})
            local = {g: j for j, g in enumerate(need)}
            per_rank[r] = {"trajs": [trajs[i] for i in need],
                           "plan": [([local[i] for i in mine], gt, ns) for mine, gt, ns in plans[r]]}
        return {
            "per_rank": per_rank, "left": set(range(dp_world)), "metrics": adv_metrics,
            "num_trajectories": len(trajs), "trained_tokens": sum(len(t.prompt_ids) + t.response_len for t in trajs),
            "response_length/mean": sum(t.response_len for t in trajs) / max(1, len(trajs)),
            "staleness/max": max((b - t.version_tag) for t in trajs) if trajs else 0,
        }

    def get_batch(self, b: int, rank: int, dp_world: int, timeout_s: float = 1800.0, tp_index: int = 0,
                  tp_size: int = 1) -> dict:
        """Data-parallel rank ``rank``'s share of staleness buffer ``b`` (blocks
        until READY).  The ``tp_size`` tensor-parallel ranks of one
        data-parallel rank all receive the same share."""
        b, rank = int(b), int(rank)
        with self._cv:
            lk = self._batch_locks.setdefault(b, threading.Lock())
        with lk:
            if b not in self._batches:
                ent = self._build(b, int(dp_world), timeout_s)
                ent["left"] = {(r, t) for r in range(int(dp_world)) for t in range(int(tp_size))}
                self._batches[b] = ent
            ent = self._batches[b]
            mine = ent["per_rank"][rank]
            ent["left"].discard((rank, int(tp_index)))
        if not ent["left"]:
            with self._cv:
                self._batches.pop(b, None)
                self._batch_locks.pop(b, None)
        out = {k: v for k, v in ent.items() if k not in ("per_rank", "left")}
        out.update(mine)
        return out

    def acquire_push(self, timeout: float = 600.0) -> bool:
        return self.ps.acquire_exclusive_push(timeout)

    def release_push(self) -> None:
        self.ps.release_exclusive_push()

    def push_model(self, version: int, locked: bool = False) -> None:
        """Publish ``version``; ``locked`` means the caller already holds the
        exclusive push lock (it wrote weight stores that rollout ranks read)."""
        if locked:
            self.ps.push_model(int(version))
            return
        if not self.ps.acquire_exclusive_push(timeout=600):
            raise TimeoutError("exclusive push lock")
        try:
            self.ps.push_model(int(version))
        finally:
            self.ps.release_exclusive_push()

    def get_ps_version(self) -> int:
        return self.ps.get_ps_model_version()

    def stats(self) -> dict:
        return {"sync": dict(self.sync_stats), "exchange": dict(self.exchange_stats),
                "manager": self.manager.snapshot(), "ps_version": self.ps.get_ps_model_version(),
                "rollout": self.rollout_summary(), "migration": dict(self.mig_stats),
                "quarantined": sorted(map(list, self.coord.quarantined))}


def _control_plane_main(cfg, vocab_size: int, n_train: int, port: int, liveness_s: float, ready=None) -> None:
    import os
    os.environ["CUDA_VISIBLE_DEVICES"] = ""        # this process never touches a GPU
    import torch
    torch.set_num_threads(1)
    cp = ControlPlane(cfg, vocab_size, n_train, liveness_s)
    server = RPCServer({"cp": cp}, port=port)
    if ready is not None:
        ready.put(int(server.address[1]))           # the port actually bound (port=0: any free one)
    try:
        cp._done.wait()
    finally:
        server.close()


def spawn_control_plane(cfg, vocab_size: int, n_train: int, port: int = 0, liveness_s: float = 300.0,
                        timeout_s: float = 600.0):
    """Start the control-plane process (rank 0 calls this once); returns
    ``(process, port)``.  With ``port=0`` the process binds a free port and
    reports it, so concurrent jobs on one machine never collide."""
    import multiprocessing as mp
    import queue
    ctx = mp.get_context("spawn")
    ready = ctx.Queue()
    p = ctx.Process(target=_control_plane_main, args=(cfg, vocab_size, n_train, port, liveness_s, ready),
                    daemon=True, name="psrl-control-plane")
    p.start()
    t0 = time.monotonic()
    while True:
        try:
            bound = ready.get(timeout=1.0)
            return p, int(bound)
        except queue.Empty:
            if not p.is_alive():
                raise RuntimeError(f"control-plane process exited with code {p.exitcode} before serving")
            if time.monotonic() - t0 > timeout_s:
                p.terminate()
                raise TimeoutError("control-plane process did not start in time")


def connect(port: int, timeout: float = 1800.0) -> RPCClient:
    c = RPCClient(("127.0.0.1", int(port)), timeout=timeout)
    return c


class ExchangeMailbox:
    """Runs a rollout instance's ``exchange`` RPCs on a background thread.

    The engine loop ``post``s finished outputs and ``collect``s the requests and
    aborts that came back; the thread batches outputs for at least
    ``min_interval`` seconds, asks for as many requests as the engine has free
    slots (minus those already received but not yet added), and keeps a
    heartbeat every ``idle_interval`` seconds even when nothing happens.
    """

    def __init__(self, proxy, instance_id, engine, min_interval: float = 0.004, idle_interval: float = 0.02):
        self.proxy = proxy
        self.instance_id = tuple(instance_id)
        self.engine = engine
        self.min_interval = float(min_interval)
        self.idle_interval = float(idle_interval)
        self.ps_version = int(engine.version)
        self.phase = 0
        self.sync_granted = False   # the coordinator's go-ahead for a weight pull
        self._tp_mark = (time.monotonic(), 0)
        self.error: BaseException | None = None
        self._lock = threading.Lock()
        self._outputs: list = []
        self._reqs: list = []
        self._aborts: list = []
        self._wake = threading.Event()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, daemon=True, name="exchange")
        self._thread.start()

    def post(self, outputs: list) -> None:
        if outputs:
            with self._lock:
                self._outputs.extend(outputs)
            self._wake.set()

    def collect(self) -> tuple[list, list]:
        with self._lock:
            reqs, aborts = self._reqs, self._aborts
            self._reqs, self._aborts = [], []
        if self.error is not None:
            raise RuntimeError("control-plane exchange failed") from self.error
        return reqs, aborts

    def kick(self) -> None:
        self._wake.set()

    def take_sync_grant(self) -> bool:
        with self._lock:
            g, self.sync_granted = self.sync_granted, False
        return g

    def _throughput(self) -> float:
        """Generated tokens per second since the previous report."""
        t0, n0 = self._tp_mark
        now, n = time.monotonic(), int(self.engine.stats.get("decode_tokens", 0))
        self._tp_mark = (now, n)
        return (n - n0) / max(now - t0, 1e-6)

    def _loop(self) -> None:
        last = 0.0
        eng = self.engine
        try:
            while not self._stop.is_set():
                self._wake.wait(self.idle_interval)
                self._wake.clear()
                if self._stop.is_set():
                    break
                dt = time.monotonic() - last
                if dt < self.min_interval:
                    time.sleep(self.min_interval - dt)
                with self._lock:
                    outs, self._outputs = self._outputs, []
                    queued = len(self._reqs)
                free = max(0, eng.max_num_seqs - eng.num_unfinished() - queued)
                state = {"running": len(eng.running), "waiting": len(eng.waiting) + queued,
                         "kv_usage": float(eng.bm.usage()), "throughput": self._throughput()}
                reqs, aborts, v, phase, sync = self.proxy.exchange(self.instance_id, eng.version, free, outs, state)
                last = time.monotonic()
                with self._lock:
                    self._reqs.extend(reqs)
                    self._aborts.extend(aborts)
                    if sync:
                        self.sync_granted = True
                self.ps_version = int(v)
                self.phase = int(phase)
        except BaseException as exc:     # surfaced to the engine loop by collect()
            self.error = exc

    def close(self) -> None:
        self._stop.set()
        self._wake.set()
        self._thread.join(timeout=30)
