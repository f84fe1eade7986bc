"""Rollout coordination in the live control plane (CPU, no GPU): the
coordinator grants weight syncs through ``ControlPlane.exchange`` (one grant
per lagging instance until it reports the new version), a failed pull
quarantines the instance, and load-balanced migration moves running requests
from a busy instance to an idle one with their generated tokens."""

from psrl_b200.config import load_config
from psrl_b200.rollout.engine import RequestOutput
from psrl_b200.trainer.control_plane import ControlPlane


def _cp(overrides=()):
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["psrl.staleness_buffer_entries=4", "psrl.staleness=2",
                                                         "actor.ppo_mini_batch_size=4", *overrides])
    cp = ControlPlane(cfg, 1024, n_train=1)
    for iid in ((0, 0), (1, 0)):
        cp.register_instance(iid, 0)
    return cfg, cp


def _state(running=0, waiting=0):
    return {"running": running, "waiting": waiting, "kv_usage": 0.1, "throughput": 100.0}


def test_sync_grant_once_per_lagging_instance():
    cfg, cp = _cp()
    *_, sync = cp.exchange((0, 0), 0, 0, [], _state())
    assert not sync                              # PS at version 0: nothing to pull
    cp.ps.push_model(1)
    *_, sync = cp.exchange((0, 0), 0, 0, [], _state())
    assert sync                                  # lagging: granted
    *_, sync = cp.exchange((0, 0), 0, 0, [], _state())
    assert not sync                              # still pulling: no second grant
    *_, sync = cp.exchange((0, 0), 1, 0, [], _state())
    assert not sync and (0, 0) not in cp.coord.syncing
    cp.report_pull(0.01, (0, 0), 0, 1, 3)
    assert cp.coord.history[-1].to_version == 1 and cp.coord.history[-1].interrupted == 3


def test_failed_pull_quarantines_instance():
    cfg, cp = _cp()
    cp.ps.push_model(1)
    cp.exchange((1, 0), 0, 0, [], _state())
    cp.report_sync_failure((1, 0), "IPC mapping lost")
    reqs, *_ = cp.exchange((1, 0), 0, 16, [], _state())
    assert reqs == []                            # no more work for a quarantined instance
    assert [1, 0] in cp.stats()["quarantined"]
    reqs, *_ = cp.exchange((0, 0), 0, 16, [], _state())
    assert reqs                                  # the healthy one keeps serving


def test_migration_moves_running_requests_to_the_idle_instance():
    cfg, cp = _cp(["psrl.rollout_coordination.sync_and_mig_strategy.mig.enable=true",
                   "psrl.rollout_coordination.sync_and_mig_strategy.mig.threshold=2.0",
                   "psrl.rollout_coordination.sync_and_mig_strategy.mig.stop_threshold=1.0",
                   "psrl.rollout_coordination.sync_and_mig_strategy.check_interval_in_ms=0"])
    busy, idle = (0, 0), (1, 0)
    reqs, *_ = cp.exchange(busy, 0, 8, [], _state())
    assert len(reqs) == 8
    cp.exchange(idle, 0, 0, [], _state(running=0))
    # the busy instance reports its load: the coordinator plans a move
    _, aborts, *_ = cp.exchange(busy, 0, 0, [], _state(running=8))
    assert aborts and cp.stats()["migration"]["requests"] == len(aborts)
    moved = set(aborts)
    # the busy engine interrupts them and returns partial outputs
    outs = [RequestOutput(r.request_id, r.prompt_ids, [7, 7], [-0.1, -0.2], [0, 0], "abort", 0, dict(r.meta))
            for r in reqs if r.request_id in moved]
    back, *_ = cp.exchange(busy, 0, len(moved), outs, _state(running=8 - len(moved)))
    assert not moved & {r.request_id for r in back}      # not handed back to the busy instance
    got, *_ = cp.exchange(idle, 0, 16, [], _state())
    resumed = {r.request_id: r for r in got if r.request_id in moved}
    assert set(resumed) == moved
    assert all(r.prev_output_ids == [7, 7] for r in resumed.values())   # tokens so far kept
    cp.ps.staleness_inventory.check_invariants()


def test_pull_dispatch_follows_routing_policy():
    """Training dispatch goes through the router in pull mode: with request-count
    balancing a loaded instance passes requests over for an idle one; with group
    stickiness every member of a prompt group lands on the group's first instance."""
    cfg, cp = _cp()
    busy, idle = (0, 0), (1, 0)
    cp.exchange(idle, 0, 0, [], _state(running=0))
    reqs, *_ = cp.exchange(busy, 0, 8, [], _state(running=40))      # far more loaded than the idle one
    assert reqs == [] and cp.manager.stats.get("routed_elsewhere", 0) > 0
    got, *_ = cp.exchange(idle, 0, 8, [], _state(running=0))
    assert len(got) == 8

    cfg, cp = _cp(["psrl.rollout_coordination.routing_strategy.enable_group_sticky=true"])
    a, b = (0, 0), (1, 0)
    cp.exchange(b, 0, 0, [], _state())
    first, *_ = cp.exchange(a, 0, 3, [], _state())                   # a takes part of the first group
    rest, *_ = cp.exchange(b, 0, 16, [], _state())                   # b must leave that group to a
    uids_a = {r.meta["uid"] for r in first}
    assert not uids_a & {r.meta["uid"] for r in rest}
