"""Rollout coordinator: weight-sync gating, migration and replica health (C16).

The coordinator watches every rollout instance and decides

* **when to sync** an instance that lags the PS version: ``greedy`` as soon as it
  lags (in-flight requests continue as partial rollouts after re-prefill), or
  ``status_based`` when its waiting queue is empty and its load indicator is at
  or below a threshold (``_check_should_sync``);
* **the sync protocol**: pause routing to the instance → pause it → interrupt
  partial requests (they loop back to the dispatcher with their tokens so far)
  → pull weights → publish the new version → resume; on failure the instance
  is quarantined (no more routing) instead of resumed (``sync_with_ps``,
  ``_finish_gateway_sync``, ``_quarantine_failed_replicas``);
* **migration**: when the ratio between the most and least loaded instances
  (by ``request_num``, ``throughput`` or ``kv_cache``) exceeds the threshold,
  move requests from the busiest instance (abort with requeue → the router
  places them elsewhere, keeping their generated tokens) until the ratio falls
  under ``stop_threshold`` (``_check_should_migrate``).

Instances are driven through a small handle interface so the same logic runs
for in-process engines and for remote rollout ranks.
Reference: ``psrl/workers/gen/rollout_coordination/``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

from .router import InstanceState


@dataclass
class SyncRecord:
    instance_id: tuple
    from_version: int
    to_version: int
    seconds: float
    interrupted: int
    ok: bool


@dataclass
class CoordinatorConfig:
    method: str = "greedy"             # greedy | status_based
    partial_rollout: bool = True
    sync_threshold: float | None = None
    sync_indicator: str = "request_num"
    mig_enable: bool = False
    mig_indicator: str = "request_num"
    mig_threshold: float = 2.0         # start when max/min load ratio exceeds this
    mig_stop_threshold: float = 1.25
    mig_max_per_round: int = 16

    @classmethod
    def from_cfg(cls, cfg) -> "CoordinatorConfig":
        sm = cfg.psrl.rollout_coordination.sync_and_mig_strategy
        mig = sm.mig
        return cls(sm.method, bool(cfg.psrl.rollout_coordination.partial_rollout.enable),
                   sm.sync.get("threshold"), sm.sync.get("indicator", "request_num"), bool(mig.enable),
                   mig.get("indicator", "request_num"), float(mig.get("threshold") or 2.0),
                   float(mig.get("stop_threshold") or 1.25))


def indicator(s: InstanceState, kind: str) -> float:
    if kind == "kv_cache":
        return s.kv_usage
    if kind == "throughput":
        return s.throughput
    return float(s.load)


class RolloutCoordinator:
    def __init__(self, cfg: CoordinatorConfig, ps_version_fn):
        self.cfg = cfg
        self.ps_version = ps_version_fn
        self.quarantined: set = set()
        self.syncing: set = set()
        self.history: list[SyncRecord] = []
        self.ready_buffers: list[int] = []
        self.migrations = 0

    # ------------------------------------------------------------------ sync
    def should_sync(self, s: InstanceState) -> bool:
        v = self.ps_version()
        if s.instance_id in self.quarantined or s.instance_id in self.syncing or v <= s.version:
            return False
        if not self.cfg.partial_rollout and s.load > 0:
            return False
        if self.cfg.method == "greedy":
            return True
        if s.num_waiting > 0:
            return False
        if self.cfg.sync_threshold is None:
            return True
        return indicator(s, self.cfg.sync_indicator) <= self.cfg.sync_threshold

    def sync_with_ps(self, handle, s: InstanceState) -> SyncRecord:
        """handle: pause(), interrupt_partial() -> int, pull(version) -> int, resume()."""
        t0 = time.perf_counter()
        target = self.ps_version()
        self.syncing.add(s.instance_id)
        s.paused = True
        ok = True
        interrupted = 0
        try:
            handle.pause()
            if self.cfg.partial_rollout:
                interrupted = handle.interrupt_partial()
            new_v = handle.pull(target)
            s.version = new_v
            handle.resume()
            s.paused = False
        except Exception:
            ok = False
            self.quarantine(s)
        finally:
            self.syncing.discard(s.instance_id)
        rec = SyncRecord(s.instance_id, s.version if not ok else s.version, target, time.perf_counter() - t0,
                         interrupted, ok)
        self.history.append(rec)
        return rec

    def quarantine(self, s: InstanceState) -> None:
        self.quarantined.add(s.instance_id)
        s.healthy = False
        s.paused = True

    def update_ready_buffer(self, buffer_id: int) -> None:
        self.ready_buffers.append(int(buffer_id))

    # ------------------------------------------------------------- migration
    def plan_migration(self, instances: list[InstanceState]) -> list[tuple[tuple, tuple, int]]:
        """(from_instance, to_instance, n_requests) moves for this round."""
        if not self.cfg.mig_enable:
            return []
        live = [s for s in instances if s.healthy and not s.paused]
        if len(live) < 2:
            return []
        kind = self.cfg.mig_indicator
        busy = max(live, key=lambda s: indicator(s, kind))
        idle = min(live, key=lambda s: indicator(s, kind))
        hi, lo = indicator(busy, kind), indicator(idle, kind)
        if hi <= self.cfg.mig_threshold * max(lo, 1e-9) or busy.instance_id == idle.instance_id:
            return []
        if kind != "request_num":
            n = max(1, int(busy.load * 0.1))
        else:
            # move until hi/lo <= stop threshold: hi - n <= stop * (lo + n)
            stop = self.cfg.mig_stop_threshold
            n = int((hi - stop * lo) / (1 + stop))
        n = max(0, min(n, self.cfg.mig_max_per_round, busy.num_running))
        if n == 0:
            return []
        self.migrations += n
        return [(busy.instance_id, idle.instance_id, n)]
