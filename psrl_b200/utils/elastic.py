"""Resource elasticity (C30): decide when shared GPUs switch between rollout and
training roles (sleep/wake of instances).

``ScalingPolicy.decide`` consumes per-instance signals (KV usage, waiting
queue, throughput) and an arrival-rate estimate:

* the load of the rollout fleet is ``rho = lambda / (mu * n_awake)`` with
  ``lambda`` the EWMA request arrival rate and ``mu`` the per-instance service
  rate from the fitted throughput curve ``A * (1 - (B x + 1) ** -k)``;
* scale **up** (wake one sleeping instance) when ``rho > theta_max`` or any
  instance is saturated (KV usage or queue), scale **down** (put one to sleep)
  when ``rho < theta_low`` and no instance has a long queue;
* a hysteresis band and a cooldown prevent flapping; at least
  ``min_awake_per_role`` instances stay awake.

``ElasticExecutor`` runs the monitor loop, applies decisions through
caller-provided ``sleep(instance)`` / ``wake(instance)`` callbacks, and
abandons a decision whose execution stalls for too many ticks.
Reference: ``psrl/utils/elastic_rm/{elastic_executor,scaling_policy}.py``.
"""

from __future__ import annotations

import threading
import time
from dataclasses import dataclass, field


@dataclass
class InstanceSignal:
    instance_id: tuple
    awake: bool
    kv_usage: float = 0.0
    num_waiting: int = 0
    num_running: int = 0
    throughput: float = 0.0


@dataclass
class ThroughputFit:
    A: float = 7271.5
    B: float = 0.05
    k: float = 1.0
    tokens_per_request: float = 1024.0

    def service_rate(self, concurrency: float) -> float:
        """requests/s one instance completes at the given concurrency."""
        tps = self.A * (1.0 - (self.B * concurrency + 1.0) ** (-self.k))
        return tps / max(1.0, self.tokens_per_request)


@dataclass
class Decision:
    action: str                  # "up" | "down" | "none"
    instance_id: tuple | None = None
    reason: str = ""


@dataclass
class ScalingPolicy:
    theta_low: float = 0.1
    theta_max: float = 0.8
    hysteresis: float = 0.05
    cooldown_ms: float = 10_000
    min_awake: int = 1
    max_waiting_for_down: int = 64
    kv_full: float = 0.95
    lambda_alpha: float = 0.2
    fit: ThroughputFit = field(default_factory=ThroughputFit)
    _lambda: float = 0.0
    _last_action_ms: float = -1e18
    _last: str = "none"

    def observe_arrivals(self, n: int, dt_s: float) -> float:
        rate = n / max(dt_s, 1e-9)
        self._lambda = self.lambda_alpha * rate + (1 - self.lambda_alpha) * self._lambda
        return self._lambda

    def decide(self, signals: list[InstanceSignal], now_ms: float | None = None) -> Decision:
        now_ms = time.monotonic() * 1000 if now_ms is None else now_ms
        if now_ms - self._last_action_ms < self.cooldown_ms:
            return Decision("none", reason="cooldown")
        awake = [s for s in signals if s.awake]
        asleep = [s for s in signals if not s.awake]
        if not awake:
            return Decision("up", asleep[0].instance_id, "no awake instance") if asleep else Decision("none")
        conc = sum(s.num_running for s in awake) / len(awake)
        mu = max(1e-9, self.fit.service_rate(max(conc, 1.0)))
        rho = self._lambda / (mu * len(awake))
        up_thr = self.theta_max + (self.hysteresis if self._last == "down" else 0.0)
        down_thr = self.theta_low - (self.hysteresis if self._last == "up" else 0.0)
        saturated = any(s.kv_usage >= self.kv_full or s.num_waiting > self.max_waiting_for_down for s in awake)
        if asleep and (rho > up_thr or saturated):
            d = Decision("up", asleep[0].instance_id, f"rho={rho:.2f}" + (" saturated" if saturated else ""))
        elif len(awake) > self.min_awake and rho < down_thr and not saturated:
            victim = min(awake, key=lambda s: (s.num_running + s.num_waiting, s.kv_usage))
            d = Decision("down", victim.instance_id, f"rho={rho:.2f}")
        else:
            return Decision("none", reason=f"rho={rho:.2f}")
        self._last_action_ms = now_ms
        self._last = d.action
        return d


class ElasticExecutor:
    def __init__(self, policy: ScalingPolicy, get_signals, sleep_fn, wake_fn, interval_ms: float = 1000,
                 abandon_stall_ticks: int = 180):
        self.policy = policy
        self.get_signals = get_signals
        self.sleep_fn = sleep_fn
        self.wake_fn = wake_fn
        self.interval = interval_ms / 1000.0
        self.abandon = abandon_stall_ticks
        self.history: list[Decision] = []
        self._stop = threading.Event()
        self._thread = None

    def tick(self) -> Decision:
        d = self.policy.decide(self.get_signals())
        if d.action == "up":
            self.wake_fn(d.instance_id)
        elif d.action == "down":
            self.sleep_fn(d.instance_id)
        if d.action != "none":
            self.history.append(d)
        return d

    def _loop(self):
        while not self._stop.is_set():
            self.tick()
            self._stop.wait(self.interval)

    def start(self):
        self._thread = threading.Thread(target=self._loop, daemon=True, name="elastic-monitor")
        self._thread.start()

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)


class EngineFleet:
    """The executor's view of real rollout engines: signals from each engine's
    scheduler state, ``sleep`` / ``wake`` through the engines' virtual-memory
    pools (:meth:`psrl_b200.rollout.engine.RolloutEngine.sleep`).

    ``engines``: instance id -> engine (built with a ``memory_pool``).
    ``on_interrupted(outputs)``: receives the in-flight requests an engine
    interrupted when it went to sleep (the agent-loop manager's ``on_complete``
    re-queues them with their partial outputs).  ``reload(instance_id, engine)``:
    called after a wake when the engine dropped its weights while asleep (sleep
    level 2), e.g. a weight pull from the parameter server.
    Reference: ``psrl/utils/elastic_rm/elastic_executor.py:517,645``.
    """

    def __init__(self, engines: dict, on_interrupted=None, keep_weights: bool = True, reload=None):
        self.engines = dict(engines)
        self.on_interrupted = on_interrupted
        self.keep_weights = keep_weights
        self.reload = reload
        self.released_bytes = 0
        self.lock = threading.Lock()

    def signals(self) -> list[InstanceSignal]:
        out = []
        for iid, e in self.engines.items():
            out.append(InstanceSignal(iid, not e.asleep, float(e.bm.usage()) if not e.asleep else 0.0,
                                      len(e.waiting), len(e.running),
                                      float(e.stats.get("decode_tokens", 0))))
        return out

    def sleep(self, instance_id) -> int:
        with self.lock:
            e = self.engines[instance_id]
            outs, freed = e.sleep(keep_weights=self.keep_weights)
            self.released_bytes += freed
        if outs and self.on_interrupted is not None:
            self.on_interrupted(outs)
        return freed

    def wake(self, instance_id) -> int:
        with self.lock:
            e = self.engines[instance_id]
            n = e.wake()
        if not self.keep_weights and self.reload is not None:
            self.reload(instance_id, e)
        return n

    def executor(self, policy: ScalingPolicy, interval_ms: float = 1000) -> ElasticExecutor:
        return ElasticExecutor(policy, self.signals, self.sleep, self.wake, interval_ms)
