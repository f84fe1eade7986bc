"""A rollout instance: one engine plus its side of the PS protocol.

``pump`` is one scheduling round: pull admitted work from the dispatcher
(reserved in the PS at this instance's weight version), apply aborts decided by
the PS, run one engine step, and report finished trajectories.  Weight sync is
decided by a :class:`SyncPolicy` (reference coordinator:
``rollout_coordination/sync_and_migrate/greedy.py:23-80`` and
``status_based.py``): *greedy* pulls as soon as the instance lags the PS
(in-flight requests continue as partial rollouts), *status_based* waits until
the instance's queue is empty and its load indicator is below a threshold.

The dispatcher and weight source are injected, so the same class runs
colocated with the trainer (direct calls) or in its own process (RPC proxies).
"""

from __future__ import annotations

import time
from typing import Callable

from .engine import RolloutEngine


class SyncPolicy:
    def __init__(self, method: str = "greedy", partial_rollout: bool = True, threshold: float | None = None,
                 indicator: str = "request_num"):
        self.method = method
        self.partial_rollout = partial_rollout
        self.threshold = threshold
        self.indicator = indicator

    def should_sync(self, engine: RolloutEngine, ps_version: int) -> bool:
        if ps_version <= engine.version:
            return False
        if not self.partial_rollout and engine.has_unfinished():
            return False
        if self.method == "greedy":
            return True
        # status_based
        if engine.waiting:
            return False
        if self.threshold is None:
            return True
        load = {"request_num": len(engine.running), "kv_cache": engine.bm.usage()}.get(self.indicator, 0)
        return load <= self.threshold


class RolloutInstance:
    def __init__(self, instance_id, engine: RolloutEngine, dispatcher, weight_puller: Callable[[int], None],
                 ps_version_fn: Callable[[], int], policy: SyncPolicy | None = None):
        self.instance_id = instance_id
        self.engine = engine
        self.dispatcher = dispatcher
        self.pull = weight_puller
        self.ps_version = ps_version_fn
        self.policy = policy or SyncPolicy()
        self.sync_count = 0
        self.sync_time = 0.0

    def admit(self) -> int:
        free = self.engine.max_num_seqs - self.engine.num_unfinished()
        if free <= 0:
            return 0
        reqs = self.dispatcher.take_work(self.instance_id, self.engine.version, free)
        for r in reqs:
            self.engine.add_request(r)
        return len(reqs)

    def apply_aborts(self) -> None:
        for rid in self.dispatcher.take_aborts(self.instance_id):
            self.engine.abort(rid)

    def maybe_sync(self) -> bool:
        v = self.ps_version()
        if not self.policy.should_sync(self.engine, v):
            return False
        t0 = time.perf_counter()
        self.pull(v)
        self.sync_time += time.perf_counter() - t0
        self.sync_count += 1
        return True

    def pump(self) -> int:
        self.maybe_sync()
        self.admit()
        self.apply_aborts()
        outs = self.engine.step()
        if outs:
            self.dispatcher.on_complete(outs, self.instance_id)
        return len(outs)
