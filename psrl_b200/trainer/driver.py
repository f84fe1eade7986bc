"""The RL driver: ``RLTrainer.fit`` / ``RLTrainer.step`` (C1/C2/C3).

One training step consumes staleness buffer ``b = global_step``:

1. wait until the buffer is READY (the rollout side keeps generating meanwhile);
2. take its trajectories, compute advantages (GRPO / GAE / ...), optionally
   recompute old log-probs, reference log-probs and values;
3. update the critic and the actor (PPO-family loss);
4. publish the new weights under the exclusive push lock and advance the PS
   version to ``b + 1`` (which lets the dispatcher release more prompts and the
   rollout instances sync).

Placement:

* **colocated** (one process / one GPU): the rollout engine and the trainer
   share the device; waiting for a buffer means running engine steps, and the
   weight sync is an in-HBM copy into the engine's fused-layout weights.
* **disaggregated** (``torch.distributed.run``, N GPUs): ranks ``[0, n_train)``
   train, the others serve rollout; see :mod:`psrl_b200.trainer.distributed`.

Reference: ``PSRL_RayPPOTrainer.fit`` (``psrl/trainer/ppo/ray_trainer.py:3127``),
``FullBatchStepStrategy.run_step`` (``psrl/trainer/ppo/strategies/full_batch.py:26``).
"""

from __future__ import annotations

import time

import torch

from ..agent.data import DataProcessor
from ..agent.manager import AgentLoopManager
from ..config import redundant_settings
from ..models import model_args_from_config
from ..ps import PSManager
from ..reward import RewardManager
from ..rollout.engine import EngineWeights, RolloutEngine
from ..rollout.instance import RolloutInstance, SyncPolicy
from ..utils.events import EventLog
from . import algos
from .actor import PolicyWorker



def trainer_stream_for(cfg, device, active: bool):
    """The stream the trainer launches on while a rollout engine runs beside
    it: a green-context stream that leaves ``psrl.deployment.rollout_reserved_sms``
    SMs to the engine, or None (the current stream)."""
    k = int(cfg.psrl.deployment.get("rollout_reserved_sms", 0) or 0)
    if not active or k <= 0 or torch.device(device).type != "cuda":
        return None
    from ..parallel.sm_partition import trainer_stream
    s, _ = trainer_stream(torch.device(device), k)
    return s


def train_stream_ctx(stream):
    import contextlib
    return torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()


def _apply_switch_interval(cfg) -> None:
    """A trainer thread that launches thousands of kernels per micro-batch holds
    the GIL for long stretches; a short switch interval bounds how long the
    rollout thread waits for it between decode steps."""
    v = cfg.trainer.get("gil_switch_interval_s")
    if v:
        import sys
        sys.setswitchinterval(float(v))

def resolve_device(cfg) -> torch.device:
    d = cfg.trainer.get("device", "auto")
    if d == "auto":
        return torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    return torch.device(d)


def compute_batch_advantages(cfg, trajs, kl_ctrl=None) -> dict:
    """Fill ``advantage`` / ``token_advantages`` / ``returns`` on the
    trajectories.  With ``kl_ctrl`` (``algorithm.use_kl_in_reward``) the
    per-token rewards first get the KL penalty against the reference policy
    (``ref_logprobs`` must be set)."""
    est = cfg.algorithm.adv_estimator
    if not trajs:
        return {}
    out = {}
    if kl_ctrl is not None:
        out.update(algos.apply_kl_in_reward(trajs, kl_ctrl, str(cfg.algorithm.get("kl_penalty", "kl"))))
    raw = torch.tensor([t.reward for t in trajs], dtype=torch.float32)
    scores = torch.tensor([algos.trajectory_score(t) for t in trajs], dtype=torch.float32)
    uids = [t.uid for t in trajs]
    if est in ("grpo", "rloo", "gdpo", "optimal_token_baseline"):
        lengths = torch.tensor([t.response_len for t in trajs])
        adv = algos.compute_advantages(est, scores=scores, uids=uids, norm_by_std=bool(cfg.algorithm.norm_adv_by_std_in_grpo),
                                       lengths=lengths, score_components=algos.score_components(trajs))
        for t, a in zip(trajs, adv.tolist()):
            t.advantage = a
            t.token_advantages = None
    else:
        L = max(t.response_len for t in trajs)
        N = len(trajs)
        rew = torch.zeros(N, L)
        mask = torch.zeros(N, L)
        vals = torch.zeros(N, L)
        for i, t in enumerate(trajs):
            n = t.response_len
            mask[i, :n] = algos.response_mask_row(t)
            rew[i, :n] = torch.tensor(algos.token_reward_row(t), dtype=torch.float32)
            if t.old_values is not None:
                vals[i, :n] = torch.tensor(t.old_values[:n])
        if est == "gae":
            adv, ret = algos.gae_advantage(rew, vals, mask, float(cfg.algorithm.gamma), float(cfg.algorithm.lam))
        else:
            adv = algos.compute_advantages(est, scores=scores, uids=uids, token_rewards=rew, mask=mask,
                                           gamma=float(cfg.algorithm.gamma))
            ret = adv
        for i, t in enumerate(trajs):
            n = t.response_len
            t.token_advantages = adv[i, :n].tolist()
            t.returns = ret[i, :n].tolist()
    out.update({"critic/score_mean": float(raw.mean()), "critic/score_max": float(raw.max()),
                "critic/score_min": float(raw.min())})
    if kl_ctrl is not None:
        out["critic/rewards_mean"] = float(scores.mean())
    return out


class RLTrainer:
    """Colocated asynchronous RL trainer (one process drives trainer and rollout)."""

    def __init__(self, cfg, device=None, seed: int | None = None, log: EventLog | None = None):
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else resolve_device(cfg)
        self.seed = int(cfg.trainer.seed if seed is None else seed)
        if log is None and cfg.trainer.get("event_log_dir", None):
            from ..utils.events import rank_event_log
            log = rank_event_log(cfg, 0, "driver")
        self.log = log or EventLog()
        self.args = model_args_from_config(cfg.model)
        rn, alg_rn, _, _ = redundant_settings(cfg)
        self.ps = PSManager.from_config(cfg)
        self.data = DataProcessor(cfg, self.args.vocab_size, rn)
        self.reward = RewardManager(cfg, self.data.tokenizer)
        self.manager = AgentLoopManager(cfg, self.ps, self.data, self.reward)
        self.actor = PolicyWorker(cfg, self.args, self.device, seed=self.seed)
        self.critic = None
        if cfg.critic.enable:
            from dataclasses import replace
            cargs = replace(self.args, value_head=True, tie_word_embeddings=False)
            self.critic = PolicyWorker(cfg, cargs, self.device, seed=self.seed + 1)
        self.ref = None
        if cfg.actor.use_kl_loss or cfg.algorithm.use_kl_in_reward:
            self.ref = PolicyWorker(cfg, self.args, self.device, seed=self.seed, trainable=False)
        self.kl_ctrl = algos.kl_controller(cfg.algorithm) if cfg.algorithm.use_kl_in_reward else None
        rc = cfg.rollout
        self.engine_weights = EngineWeights.from_model(self.actor.model, self.device, dtype=self.actor.dtype)
        max_len = int(rc.max_prompt_length) + int(rc.max_response_length) + 64
        # time sharing without overlap (rollout.enable_sleep_mode): the engine's
        # KV cache and weights live in virtual-memory regions, released while
        # the trainer trains and mapped back before the next generation phase
        pool = None
        if bool(rc.get("enable_sleep_mode", False)) and self.device.type == "cuda":
            from ..parallel.memory import MemoryPool
            pool = MemoryPool(self.device)
        self.engine = RolloutEngine(
            self.args, self.engine_weights, memory_pool=pool, max_num_seqs=int(rc.max_num_seqs), max_model_len=max_len,
            block_size=int(rc.block_size), max_num_batched_tokens=int(rc.max_num_batched_tokens),
            kv_cache_gb=float(rc.get("kv_cache_gb", 4.0)), enable_prefix_caching=bool(rc.enable_prefix_caching),
            use_cuda_graph=bool(rc.cuda_graph), keep_kv_on_update=bool(cfg.psrl.rollout_coordination.partial_rollout.get("keep_kv", False)),
            eos_token_id=self.data.tokenizer.eos_id if not rc.ignore_eos else None, decode_gemm=str(cfg.rollout.get("decode_gemm", "library")),
            kv_offload_blocks=int(cfg.rollout.get("kv_offload_blocks", 0) or 0))
        sm = cfg.psrl.rollout_coordination.sync_and_mig_strategy
        policy = SyncPolicy(sm.method, bool(cfg.psrl.rollout_coordination.partial_rollout.enable),
                            sm.sync.get("threshold"), sm.sync.get("indicator", "request_num"))
        self.instance_id = (0, 0)
        self.ps.register_rollout_instance(self.instance_id, 0)
        self.instance = RolloutInstance(self.instance_id, self.engine, self.manager, self._pull_weights,
                                        self.ps.get_ps_model_version, policy)
        self.global_step = 0
        self.trained_tokens = 0
        # overlapped colocation: the engine runs in its own thread on a high-priority
        # stream while the trainer trains (bounded by the staleness protocol)
        self.overlap = bool(cfg.psrl.deployment.get("colocate_overlap", True)) and self.device.type == "cuda"
        self._rollout_thread = None
        self._rollout_stop = False
        self._rollout_error: BaseException | None = None
        self.rollout_stream = torch.cuda.Stream(device=self.device, priority=-1) if self.overlap else None
        self.train_stream = trainer_stream_for(cfg, self.device, self.overlap)
        _apply_switch_interval(cfg)
        from .strategies import build_step_strategy
        self.strategy = build_step_strategy(self)

    # ----------------------------------------------------------- weights
    @torch.no_grad()
    def _pull_weights(self, version: int) -> None:
        if not self.ps.acquire_shared_pull(timeout=600):
            raise TimeoutError("could not take the shared pull lock")
        try:
            v, _ = self.ps.pull_model(self.instance_id)
            src = dict(self.actor.model.named_parameters())
            src.update(dict(self.actor.model.named_buffers()))
            for k, t in self.engine_weights.tensors.items():
                if k in src:
                    t.copy_(src[k].detach(), non_blocking=True)
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            self.engine.load_weights(None, v)
        finally:
            self.ps.release_shared_pull()

    # ------------------------------------------------------- rollout thread
    def _rollout_loop(self) -> None:
        try:
            with torch.cuda.stream(self.rollout_stream):
                while not self._rollout_stop:
                    self.instance.pump()
                    if not self.engine.has_unfinished():
                        time.sleep(0.0005)
        except BaseException as exc:  # surfaced to the trainer thread
            self._rollout_error = exc

    def start_rollout(self) -> None:
        if self.overlap and self._rollout_thread is None:
            import atexit
            import threading
            import weakref
            self._rollout_stop = False
            ref = weakref.ref(self)
            # never leave the engine thread running CUDA work into interpreter shutdown
            atexit.register(lambda: ref() is not None and ref().stop_rollout())
            self._rollout_thread = threading.Thread(target=self._rollout_loop, daemon=True, name="rollout")
            self._rollout_thread.start()

    def stop_rollout(self) -> None:
        if self._rollout_thread is not None:
            self._rollout_stop = True
            self._rollout_thread.join()
            self._rollout_thread = None

    def _push_guard(self):
        import contextlib

        @contextlib.contextmanager
        def guard():
            if not self.ps.acquire_exclusive_push(timeout=600):
                raise TimeoutError("could not take the exclusive push lock")
            try:
                yield
            finally:
                self.ps.release_exclusive_push()
        return guard

    def _publish(self, version: int) -> None:
        if not self.ps.acquire_exclusive_push(timeout=600):
            raise TimeoutError("could not take the exclusive push lock")
        try:
            self.ps.push_model(version)
        finally:
            self.ps.release_exclusive_push()

    # -------------------------------------------------------------- step
    def wait_for_buffer(self, b: int, timeout_s: float = 3600.0) -> None:
        t0 = time.monotonic()
        t_act = t0
        if self.overlap:
            self.start_rollout()
        while not self.manager.buffer_ready(b):
            if time.monotonic() - t_act > self.manager.filter_patience_s:
                t_act = time.monotonic()
                self.manager.handle_waiting_buffer(b)
            if self.overlap:
                if self._rollout_error is not None:
                    raise RuntimeError("rollout thread failed") from self._rollout_error
                time.sleep(0.002)
            else:
                self.instance.pump()
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"buffer {b} not ready after {timeout_s}s: {self.manager.snapshot()}")
        if not self.overlap and self.engine.pool is not None:
            # generation phase over: hand the GPU memory to the trainer; in-flight
            # requests go back to the dispatcher as partial rollouts
            outs, freed = self.engine.sleep(keep_weights=False)
            if outs:
                self.manager.on_complete(outs, self.instance_id)
            self.log.emit("engine sleep", "SWITCH", freed_bytes=int(freed))

    def step(self) -> dict:
        b = self.global_step
        if not hasattr(self, "obs"):
            from ..utils.profiling import StepObserver
            self.obs = StepObserver(self.cfg, self.device, 0)
        self.obs.begin(b)
        metrics: dict = {}
        t0 = time.perf_counter()
        with train_stream_ctx(self.train_stream):
            trajs = self.strategy.run_step(b, metrics)
        with self.log.span("PUSH", step=b):
            self._publish(b + 1)
        if self.engine.asleep:
            self.engine.wake()
            self._pull_weights(b + 1)    # the weights were dropped while asleep
        self.global_step += 1
        ntok = sum(len(t.prompt_ids) + t.response_len for t in trajs)
        self.trained_tokens += ntok
        metrics.update({
            "step": b, "num_trajectories": len(trajs), "trained_tokens": ntok,
            "response_length/mean": sum(t.response_len for t in trajs) / max(1, len(trajs)),
            "timing_s/step": time.perf_counter() - t0,
            "ps_version": self.ps.get_ps_model_version(),
            "staleness/max": max((b - t.version_tag) for t in trajs) if trajs else 0,
        })
        metrics.update({f"rollout/{k}": v for k, v in self.engine.engine_stats().items() if isinstance(v, (int, float))})
        from .perf import perf_metrics
        metrics.update(perf_metrics(self.cfg, self.args, ntok, len(trajs), metrics["timing_s/step"],
                                    float(metrics.get("timing_s/train", 0.0)), 1, 1))
        self.obs.end(b, metrics)
        path = self.cfg.trainer.get("engine_stats_path", None)
        if path:
            from ..rollout.stats import EngineStats, StatsRecorder, ThroughputWindow
            if not hasattr(self, "_stats_rec"):
                self._stats_rec, self._stats_win = StatsRecorder(str(path)), ThroughputWindow()
            self._stats_rec.record(EngineStats.from_engine(self.instance_id, self.engine, self._stats_win))
        return metrics

    def fit(self, num_steps: int | None = None) -> list[dict]:
        if self.cfg.trainer.resume_mode != "disable" and self.global_step == 0:
            self.resume()
        # trainer.total_training_steps counts from step 0: a resumed run does the rest
        n = int(num_steps) if num_steps is not None else \
            max(0, int(self.cfg.trainer.total_training_steps) - self.global_step)
        out = []
        for _ in range(n):
            out.append(self.step())
            freq = int(self.cfg.trainer.save_freq)
            if freq > 0 and self.global_step % freq == 0:
                self.save_checkpoint()
            tf = int(self.cfg.trainer.get("test_freq", -1))
            if tf > 0 and self.global_step % tf == 0:
                out[-1].update(self.validate())
        self.manager.flush_turn_records()
        return out

    # --------------------------------------------------------- validation
    VAL_RID_BASE = 1 << 50

    def validate(self, num_prompts: int | None = None) -> dict:
        """Generate on the validation prompts with the current weights and
        score them (``val/score_mean``, ``val/response_length/mean``).

        The rollout engine is shared with training: the overlapped rollout
        thread is paused, validation requests join the in-flight training
        requests (whose completions still go to the agent-loop manager), and
        generation continues until every validation request finished.  The
        engine first pulls the latest published weights.  Validation samples
        use ``trainer.val_temperature`` (0 = greedy) and ``psrl.val_rollout_n``
        samples per prompt.  Reference: the trainer's validate step
        (``psrl/trainer/ppo/ray_trainer.py``, ``test_freq``)."""
        from ..rollout.engine import GenRequest, SamplingParams
        from .batch import Trajectory
        self.stop_rollout()
        cfg = self.cfg
        n = int(num_prompts if num_prompts is not None else cfg.data.get("val_size", 32))
        per = max(1, int(cfg.psrl.get("val_rollout_n", 1)))
        temp = float(cfg.trainer.get("val_temperature", 0.0))
        rc = cfg.rollout
        ps_v = self.ps.get_ps_model_version()
        if ps_v > self.engine.version:
            self._pull_weights(ps_v)
        items = self.data.validation_items(n)
        pending: dict[int, tuple] = {}
        for i, it in enumerate(items):
            for j in range(per):
                rid = self.VAL_RID_BASE + i * per + j
                mt = int(it.response_lens[j % len(it.response_lens)]) if it.response_lens else int(rc.max_response_length)
                params = SamplingParams(temperature=temp, top_p=1.0, top_k=-1, max_tokens=mt,
                                        ignore_eos=bool(rc.ignore_eos), seed=rid)
                meta = dict(it.meta)
                if it.answer is not None:
                    meta["answer"] = it.answer
                self.engine.add_request(GenRequest(rid, list(it.prompt_ids), params, self.engine.version, meta))
                pending[rid] = (it, meta)
        scores, lens = [], []
        ctx = torch.cuda.stream(self.rollout_stream) if self.rollout_stream is not None else None
        import contextlib
        with ctx or contextlib.nullcontext():
            while pending:
                outs = self.engine.step()
                train_outs = []
                for o in outs:
                    if o.request_id in pending:
                        it, meta = pending.pop(o.request_id)
                        tr = Trajectory(uid=it.uid, request_id=o.request_id, prompt_ids=list(o.prompt_ids),
                                        response_ids=list(o.output_ids), rollout_logprobs=list(o.logprobs),
                                        meta=meta)
                        scores.append(float(self.reward.score(tr)["score"]))
                        lens.append(len(o.output_ids))
                    else:
                        train_outs.append(o)
                if train_outs:
                    self.manager.on_complete(train_outs, self.instance_id)
        m = len(scores)
        return {"val/score_mean": sum(scores) / max(1, m), "val/response_length/mean": sum(lens) / max(1, m),
                "val/num_samples": m}

    # -------------------------------------------------------- checkpoints
    def save_checkpoint(self) -> str:
        from ..utils.checkpoint import save_checkpoint
        extra = {"kl_coef": self.kl_ctrl.value} if self.kl_ctrl is not None else {}
        return save_checkpoint(self.cfg.trainer.default_local_dir, self.global_step, self.actor, self.data,
                               self.critic, self.ps.get_ps_model_version(),
                               use_dcp=bool(self.cfg.psrl.checkpoint.use_dcp_save), extra=extra)

    def resume(self, step: int | None = None) -> int:
        """Load weights/optimizer/data cursor and re-seat the PS at that version."""
        from ..utils.checkpoint import find_latest, load_checkpoint
        root = self.cfg.trainer.get("resume_from_path") or self.cfg.trainer.default_local_dir
        if step is None and find_latest(root) is None:
            return 0
        extra: dict = {}
        step = load_checkpoint(root, self.actor, self.data, self.critic, step,
                               use_dcp=bool(self.cfg.psrl.checkpoint.use_dcp_save), extra_out=extra)
        if self.kl_ctrl is not None and "kl_coef" in extra:
            self.kl_ctrl.value = float(extra["kl_coef"])
        self.global_step = step
        self.ps.init_model_version_for_resume(step + 1)
        self.manager.initial_ps_version = step
        self.manager.request_counter = 0
        self._pull_weights(self.ps.get_ps_model_version())
        return step
