"""Host-side failure injection in the rollout plane (no GPU): a reward /
environment step that raises, an engine request that comes back as an error,
a trajectory that never finishes, a buffer stuck a few entries short.

Each test drives the agent-loop manager directly with a fake rollout instance
that takes work at version 0 and answers with fixed-length outputs, then
checks that the buffer still becomes READY with complete groups and that the
staleness inventory's invariants hold."""

import time

import pytest

from psrl_b200.agent.data import DataProcessor
from psrl_b200.agent.manager import AgentLoopManager
from psrl_b200.agent.terminate import TerminateReason
from psrl_b200.config import load_config
from psrl_b200.ps import PSManager
from psrl_b200.reward.functions import RewardManager
from psrl_b200.rollout.engine import RequestOutput


class FlakyReward:
    """Raises for the listed request ids (a failing scorer / environment),
    `times` times each, then scores like the wrapped reward."""

    def __init__(self, inner, fail_ids, times=1, exc=RuntimeError):
        self.inner, self.fail = inner, {r: times for r in fail_ids}
        self.exc = exc

    def score(self, traj):
        left = self.fail.get(traj.request_id, 0)
        if left:
            self.fail[traj.request_id] = left - 1
            raise self.exc(f"injected failure for request {traj.request_id}")
        return self.inner.score(traj)


def _setup(overrides=(), fail_ids=(), times=1, exc=RuntimeError):
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["psrl.staleness_buffer_entries=4", "psrl.staleness=1",
                                                         "actor.ppo_mini_batch_size=4",
                                                         *overrides])
    ps = PSManager.from_config(cfg)
    data = DataProcessor(cfg, 1024, int(cfg.psrl.rollout_n))
    reward = FlakyReward(RewardManager(cfg, data.tokenizer), fail_ids, times, exc)
    ps.register_rollout_instance("inst0", 0)
    return cfg, ps, AgentLoopManager(cfg, ps, data, reward)


def _pump(mgr, rounds=50, finish=lambda req: "length", skip=lambda req: False):
    """One fake instance at version 0: take work, answer it (requests for which
    ``skip`` is true are held, never answered, until the manager aborts them)."""
    held = mgr.__dict__.setdefault("_test_held", {})
    for _ in range(rounds):
        reqs = mgr.take_work("inst0", 0, 64)
        outs = []
        for r in reqs:
            if skip(r):
                held[r.request_id] = r
                continue
            n = 3
            outs.append(RequestOutput(r.request_id, r.prompt_ids, [5] * n, [-0.5] * n, [0] * n, finish(r),
                                      r.version_tag, dict(r.meta)))
        for rid in mgr.take_aborts("inst0"):
            req = held.pop(rid, None) or next((x for x in reqs if x.request_id == rid), None)
            if req is not None:
                outs.append(RequestOutput(rid, req.prompt_ids, [], [], [], "abort", req.version_tag, dict(req.meta)))
        mgr.on_complete(outs, "inst0")
        if mgr.buffer_ready(0):
            return True
    return mgr.buffer_ready(0)


def _pump_until(mgr, cond, rounds=50, **kw):
    for _ in range(rounds):
        _pump(mgr, rounds=1, **kw)
        if cond():
            return True
    return cond()


def _check_full_groups(mgr, cfg):
    trajs = mgr.consume(0)
    n = int(cfg.psrl.rollout_n)
    assert len(trajs) == 4 * n
    by_uid = {}
    for t in trajs:
        by_uid.setdefault(t.uid, []).append(t)
    assert all(len(v) == n for v in by_uid.values())
    mgr.ps.staleness_inventory.check_invariants()
    return by_uid


def test_terminate_reason_classes():
    R = TerminateReason
    assert R.ROLLOUT_ERROR.needs_worker_retry() and R.ROLLOUT_ERROR.needs_manager_retry()
    assert R.ENV_TIMEOUT.needs_worker_retry() and not R.ENV_TIMEOUT.needs_manager_retry()
    assert R.TRAJECTORY_TIMEOUT.needs_manager_retry()
    assert not R.FINISHED.needs_worker_retry() and R.FINISHED.is_successful
    assert R.ABORTED.is_aborted and not R.ABORTED.needs_manager_retry()


def test_worker_retry_recovers_a_flaky_trajectory():
    cfg, ps, mgr = _setup(["rollout.agent.retry_limit=2"], fail_ids=[1], times=1)
    assert _pump(mgr)
    assert mgr.stats["retried_trajs"] == 1 and mgr.stats["failed_groups"] == 0
    by_uid = _check_full_groups(mgr, cfg)
    # the flaky request's group completes after the retry (in this buffer or a later one)
    for _ in range(10):
        if 0 in by_uid or 0 in mgr.store:
            break
        _pump(mgr, rounds=1)
    assert 0 in by_uid or 0 in mgr.store
    assert 0 not in mgr.failed_groups


def test_manager_retry_replaces_a_group_that_keeps_failing():
    cfg, ps, mgr = _setup(["rollout.agent.retry_limit=2"], fail_ids=[1], times=10)
    assert _pump_until(mgr, lambda: 0 in mgr.failed_groups and mgr.buffer_ready(0))
    assert mgr.stats["failed_groups"] == 1 and mgr.stats["retried_groups"] >= 1
    by_uid = _check_full_groups(mgr, cfg)
    # the failing group was dropped for good and a fresh prompt filled its slot
    assert 0 not in by_uid and 0 not in mgr.store and 0 in mgr.failed_groups
    assert "injected failure" in mgr.last_error


def test_manager_retry_can_be_turned_off():
    cfg, ps, mgr = _setup(["psrl.agentic_rl.manager_retry_on_error=false"], fail_ids=[2], times=10)
    with pytest.raises(RuntimeError, match="manager_retry_on_error"):
        _pump(mgr)


def test_env_timeout_drops_only_the_member():
    # an environment timeout is retried by the worker but never refills the group slot
    cfg, ps, mgr = _setup(["rollout.agent.retry_limit=1"], fail_ids=[1], times=10, exc=TimeoutError)
    assert _pump_until(mgr, lambda: mgr.stats["dropped_trajs"] >= 1 and mgr.buffer_ready(0))
    assert mgr.stats["failed_groups"] == 0
    mgr.ps.staleness_inventory.check_invariants()


def test_engine_error_output_is_retried():
    seen = set()

    def finish(req):
        if req.request_id == 3 and 3 not in seen:
            seen.add(3)
            return "error"
        return "length"

    cfg, ps, mgr = _setup(["rollout.agent.retry_limit=2"])
    assert _pump_until(mgr, lambda: mgr.stats["retried_trajs"] == 1 and mgr.buffer_ready(0), finish=finish)
    _check_full_groups(mgr, cfg)


def test_trajectory_timeout_aborts_and_refills():
    cfg, ps, mgr = _setup(["rollout.agent.trajectory_timeout_s=0.05", "rollout.agent.retry_limit=1"])
    # request 2 never answers: the manager aborts it as a trajectory timeout
    hung = {2}

    def skip(req):
        return req.request_id in hung

    for _ in range(40):
        _pump(mgr, rounds=1, skip=skip)
        if 0 in mgr.failed_groups and mgr.buffer_ready(0):
            break
        time.sleep(0.02)
    assert mgr.stats["timed_out_trajs"] >= 1
    assert mgr.stats["failed_groups"] == 1
    assert mgr.buffer_ready(0)
    _check_full_groups(mgr, cfg)


def _stuck_buffer(method):
    """Staleness 0: the four groups of buffer 0 are all the work the dispatcher
    may release; one of them never finishes, so buffer 0 stays one entry short."""
    cfg, ps, mgr = _setup([f"psrl.rollout_coordination.proactive_filter_strategy.method={method}",
                           "psrl.rollout_coordination.proactive_filter_strategy.threshold=1", "psrl.staleness=0"])
    n = int(cfg.psrl.rollout_n)
    stuck = 0
    assert not _pump(mgr, rounds=8, skip=lambda r: r.request_id // n == stuck)
    return cfg, ps, mgr, n, stuck


def test_waiting_buffer_truncate_releases_partial_buffer():
    cfg, ps, mgr, n, stuck = _stuck_buffer("truncate")
    assert mgr.handle_waiting_buffer(0)
    assert mgr.stats["truncated_buffers"] == 1
    assert mgr.buffer_ready(0)
    trajs = mgr.consume(0)
    assert stuck not in {t.uid for t in trajs}
    assert len(trajs) == 3 * n
    mgr.ps.staleness_inventory.check_invariants()


def test_waiting_buffer_retry_needs_donor_entries():
    # no later buffer holds committed entries that could move in: nothing changes
    cfg, ps, mgr, n, stuck = _stuck_buffer("retry")
    assert not mgr.handle_waiting_buffer(0)
    assert mgr.stats["waiting_buffer_moves"] == 0
    assert not mgr.buffer_ready(0)


def test_waiting_buffer_retry_moves_later_entries():
    """Buffer 0 one entry short while buffer 1 holds a committed group that may
    also land in buffer 0: the reservation is aborted, that group moves in and a
    fresh prompt is dispatched for the aborted one."""
    from psrl_b200.ps import EntryCategory
    from psrl_b200.ps.staleness import EntryInfo
    cfg, ps, mgr, n, stuck = _stuck_buffer("retry")
    inv = ps.staleness_inventory
    # a finished version-0 group parked in buffer 1 (what occupy does once buffer 0
    # has no free slot), with its trajectories in the manager's store
    inv.ensure_buffer_exists(1)
    donor = 999
    info = EntryInfo("inst0", donor, list(range(n)), 0)
    template = next(iter(mgr.store.values()))
    mgr.store[donor] = [type(t)(**{**t.__dict__, "uid": donor, "request_id": donor * n + i})
                        for i, t in enumerate(template)]
    inv._place(1, inv.buffers[1].get_first_non_occupied(), EntryCategory.OCCUPIED, info)
    before = mgr.stats["dispatched_groups"]
    assert mgr.handle_waiting_buffer(0)
    assert mgr.stats["waiting_buffer_moves"] == 1
    assert mgr.stats["dispatched_groups"] == before + 1      # fresh prompt for the aborted group
    assert mgr.buffer_ready(0)
    trajs = mgr.consume(0)
    assert stuck not in {t.uid for t in trajs} and donor in {t.uid for t in trajs}
    mgr.ps.staleness_inventory.check_invariants()
