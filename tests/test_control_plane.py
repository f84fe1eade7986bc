"""Control-plane components: router policies, coordinator decisions, PS RPC
surface, storage plans, locks, limiters, sample store, post-processors, stats."""

import threading
import time

import pytest
import torch

from psrl_b200.ps import PSManager
from psrl_b200.ps.service import PSManagerService
from psrl_b200.ps.storage import (
    BinaryTreeBroadcastPlan,
    PSStoragePlan,
    cast_train_to_gen,
    dequantize_fp8_blockwise,
    quantize_fp8_blockwise,
)
from psrl_b200.rollout.coordinator import CoordinatorConfig, RolloutCoordinator
from psrl_b200.rollout.engine import GenRequest, SamplingParams
from psrl_b200.rollout.router import InstanceState, PrefixIndex, Router
from psrl_b200.utils.concurrency import FileSlotLimiter, TokenBucket
from psrl_b200.utils.locks import exclusive_push_model_context, shared_pull_model_context, wait_for_version
from psrl_b200.utils.sample_store import SampleStore


def _req(rid, prompt=(1, 2, 3), tag=-1, **meta):
    return GenRequest(rid, list(prompt), SamplingParams(), tag, {"uid": rid // 4, **meta})


def _insts(loads, versions=None):
    versions = versions or [0] * len(loads)
    return [InstanceState((i, 0), v, num_running=l) for i, (l, v) in enumerate(zip(loads, versions))]


def test_router_request_num_balance_and_version_filter():
    r = Router("request_num_balance")
    s = r.route(_req(0), _insts([5, 1, 3]))
    assert s.instance_id == (1, 0)
    # a request tagged with version 2 cannot go to a version-1 instance
    s = r.route(_req(1, tag=2), _insts([0, 9], versions=[1, 2]))
    assert s.instance_id == (1, 0)
    assert r.route(_req(2, tag=5), _insts([0, 0])) is None


def test_router_sticky_and_round_robin_and_random():
    r = Router("round_robin")
    picks = [r.route(_req(i * 4), _insts([0, 0, 0])).instance_id for i in range(3)]
    assert picks == [(0, 0), (1, 0), (2, 0)]
    r = Router("request_num_balance")
    s = r.route(_req(7, sticky_instance=(2, 0)), _insts([0, 0, 50]))
    assert s.instance_id == (2, 0)
    r = Router("random", seed=1)
    assert r.route(_req(8), _insts([0, 0])) is not None


def test_router_group_sticky():
    r = Router("request_num_balance", group_sticky=True)
    a = r.route(_req(4), _insts([0, 1]))
    b = r.route(_req(5), _insts([10, 0]))        # same uid (1) -> same home
    assert a.instance_id == b.instance_id == (0, 0)


def test_router_cache_aware_prefix_and_balance():
    r = Router("cache_aware", block_size=4, balance_abs_threshold=100)
    toks = list(range(40))
    first = r.route(_req(0, prompt=toks), _insts([0, 0]))
    second = r.route(_req(8, prompt=toks + [99, 98]), _insts([0, 0]))
    assert second.instance_id == first.instance_id
    idx = PrefixIndex(4)
    idx.insert(toks)
    assert idx.match(toks + [1]) == 40
    # imbalance overrides cache affinity
    r2 = Router("cache_aware", block_size=4, balance_abs_threshold=2, balance_rel_threshold=1.1)
    r2.route(_req(0, prompt=toks), _insts([0, 0]))
    s = r2.route(_req(8, prompt=toks), [InstanceState((0, 0), 0, num_running=50), InstanceState((1, 0), 0)])
    assert s.instance_id == (1, 0)


def test_router_throughput_and_admission():
    ps = PSManager(staleness=0, staleness_buffer_entries=1, rollout_n=1)
    ps.register_rollout_instance((0, 0), 0)
    ps.register_rollout_instance((1, 0), 0)
    ps.add_request([0, 1])
    ps.reserve_rollout_instance_requests((0, 0), 0, 0)        # buffer 0 full (1 entry)
    r = Router("throughput_optimal", ps=ps)
    # request 1 at version 0 has no admissible buffer (staleness 0, buffer 0 reserved)
    assert r.route(_req(1), _insts([0, 0])) is None
    r2 = Router("throughput_optimal")
    assert r2.route(_req(2), _insts([100, 1])).instance_id == (1, 0)


def test_coordinator_sync_policies_and_quarantine():
    v = {"ps": 3}
    c = RolloutCoordinator(CoordinatorConfig(method="greedy"), lambda: v["ps"])
    s = InstanceState((0, 0), version=2, num_running=5)
    assert c.should_sync(s)
    c2 = RolloutCoordinator(CoordinatorConfig(method="status_based", sync_threshold=2), lambda: v["ps"])
    assert not c2.should_sync(InstanceState((0, 0), 2, num_running=5))
    assert not c2.should_sync(InstanceState((0, 0), 2, num_running=1, num_waiting=1))
    assert c2.should_sync(InstanceState((0, 0), 2, num_running=1))
    c3 = RolloutCoordinator(CoordinatorConfig(partial_rollout=False), lambda: v["ps"])
    assert not c3.should_sync(InstanceState((0, 0), 2, num_running=1))

    class H:
        def __init__(self, fail=False):
            self.fail = fail
            self.calls = []

        def pause(self):
            self.calls.append("pause")

        def interrupt_partial(self):
            self.calls.append("interrupt")
            return 3

        def pull(self, version):
            if self.fail:
                raise RuntimeError("pull failed")
            self.calls.append("pull")
            return version

        def resume(self):
            self.calls.append("resume")

    h = H()
    rec = c.sync_with_ps(h, s)
    assert rec.ok and s.version == 3 and h.calls == ["pause", "interrupt", "pull", "resume"] and not s.paused
    s2 = InstanceState((1, 0), version=1)
    rec = c.sync_with_ps(H(fail=True), s2)
    assert not rec.ok and (1, 0) in c.quarantined and not s2.healthy
    assert not c.should_sync(s2)


def test_coordinator_migration_plan():
    c = RolloutCoordinator(CoordinatorConfig(mig_enable=True, mig_threshold=2.0, mig_stop_threshold=1.0), lambda: 0)
    moves = c.plan_migration(_insts([40, 4]))
    assert moves and moves[0][0] == (0, 0) and moves[0][1] == (1, 0)
    n = moves[0][2]
    assert 0 < n <= 16
    assert c.plan_migration(_insts([10, 8])) == []


def test_ps_service_envelope():
    ps = PSManager(staleness=1, staleness_buffer_entries=2, rollout_n=2)
    ps.register_rollout_instance((0, 0), 0)
    svc = PSManagerService(ps)
    ps.add_request([0, 1])
    assert svc.CanReserveRequest([0], [0]) == {"ok": True, "result": [[True]]}
    r = svc.ReserveRolloutInstanceRequests([(0, 0)], [0], [0])
    assert r["ok"] and r["result"][0] == [1]
    assert svc.GetReserveIndicator(1, [0])["result"] == [float("-inf")]
    assert svc.UpdateRequestStatus([0], "ROLLOUT_RUNNING", 0, (0, 0))["ok"]
    bad = svc.ReserveRolloutInstanceRequests([(9, 9)], [1], [0])
    assert not bad["ok"] and "not registered" in bad["error"]
    assert svc.GetPSModelVersion()["result"] == 0


def test_storage_plan_and_broadcast_rounds():
    p = PSStoragePlan(total=1000, n_shards=3)
    assert [p.shard_range(i) for i in range(3)] == [(0, 334), (334, 668), (668, 1000)]
    assert p.owner_of(500) == 1
    for n in (1, 2, 5, 8, 13):
        plan = BinaryTreeBroadcastPlan(n)
        have = {0}
        for rnd in plan.rounds():
            for src, dst in rnd:
                assert src in have and dst not in have
            have |= {d for _, d in rnd}
        assert have == set(range(n))
        assert len(plan.rounds()) == plan.num_rounds()


def test_fp8_blockwise_cast_roundtrip():
    w = torch.randn(300, 520) * 0.02
    q, s = quantize_fp8_blockwise(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (3, 5)
    err = (dequantize_fp8_blockwise(q, s) - w).abs().max() / w.abs().max()
    assert err < 0.07
    g = cast_train_to_gen({"a.weight": w, "norm": torch.ones(8)}, "fp8")
    assert "a.weight.scale_inv" in g and g["norm"].dtype == torch.bfloat16


def test_lock_contexts_and_version_waiter():
    ps = PSManager(staleness=0, staleness_buffer_entries=1, rollout_n=1)
    with shared_pull_model_context(ps):
        assert ps.lock_state() == (False, 1)
        assert not ps.acquire_exclusive_push(timeout=0.05)
    done = []

    def pusher():
        with exclusive_push_model_context(ps):
            done.append(1)
            ps.push_model(1)
    th = threading.Thread(target=pusher)
    th.start()
    th.join(2)
    assert done and ps.lock_state() == (False, 0)
    assert wait_for_version(ps.get_ps_model_version, 1, timeout=1) == 1
    with pytest.raises(TimeoutError):
        wait_for_version(ps.get_ps_model_version, 5, timeout=0.05)


def test_limiters(tmp_path):
    lim = FileSlotLimiter(str(tmp_path), 2)
    with lim.slot() as a:
        with lim.slot() as b:
            assert a != b
            with pytest.raises(TimeoutError):
                with lim.slot(timeout=0.05):
                    pass
    tb = TokenBucket(rate_per_s=100.0, capacity=2)
    assert tb.try_acquire() and tb.try_acquire() and not tb.try_acquire()
    time.sleep(0.03)
    assert tb.try_acquire()


def test_sample_store():
    st = SampleStore()
    meta = st.kv_batch_put([1, 2], [{"x": 1}, {"x": 2, "y": 3}], tags=["a", "b"])
    assert st.kv_batch_get(meta, ["x"]) == [{"x": 1}, {"x": 2}]
    assert st.kv_clear([1]) == 1 and st.kv_list() == ["2"] and len(st) == 1


def test_post_processors():
    from psrl_b200.agent.post_process import BUFFER_PROCESSORS, GROUP_PROCESSORS
    from psrl_b200.trainer.batch import Trajectory

    def t(uid, r):
        return Trajectory(uid, 0, [1], [2], [0.0], reward=r, meta={"reward_extra": {"acc": r}})
    assert not GROUP_PROCESSORS["dynamic_sampling_filter"]([t(0, 1.0), t(0, 1.0)])
    assert GROUP_PROCESSORS["dynamic_sampling_filter"]([t(0, 1.0), t(0, 0.0)])
    kept = BUFFER_PROCESSORS["dynamic_sampling_filter"]([t(0, 1.0), t(0, 1.0), t(1, 0.0), t(1, 1.0)])
    assert {x.uid for x in kept} == {1}


def test_engine_stats_recorder_and_zmq(tmp_path):
    from psrl_b200.rollout.stats import EngineStats, StatsRecorder, ZMQPullQueue, ZMQPushQueue
    rec = StatsRecorder(str(tmp_path / "s.jsonl"))
    rec.record(EngineStats((1, 0), 3, 2, 5, 0.5))
    assert rec.read()[0]["num_running"] == 5
    pull = ZMQPullQueue("ipc://" + str(tmp_path / "q"))
    push = ZMQPushQueue("ipc://" + str(tmp_path / "q"))
    push.put(EngineStats((2, 0)).to_dict())
    got = pull.get(2000)
    assert got["instance_id"] == (2, 0)
    push.close()
    pull.close()


def test_placement_roles():
    from psrl_b200.config import load_config
    from psrl_b200.parallel.placement import Role, plan_placement
    cfg = load_config(preset="dapo_qwen2.5_3b")
    p = plan_placement(8, cfg.psrl.deployment)
    assert p.train_ranks == [0, 1, 2, 3] and len(p.instances) == 4 and p.role_of(5) is Role.Rollout
    assert plan_placement(1, cfg.psrl.deployment).colocated
    cfg7 = load_config(preset="ppo_qwen2.5_7b")
    p = plan_placement(8, cfg7.psrl.deployment)
    assert [i.ranks for i in p.instances] == [[4, 5], [6, 7]]
    cfg7.psrl.deployment.heterogeneous_rollout.enable = True
    cfg7.psrl.deployment.heterogeneous_rollout.tensor_model_parallel_size_per_instance = [1, 1, 2]
    p = plan_placement(8, cfg7.psrl.deployment)
    assert [i.tp for i in p.instances] == [1, 1, 2] and p.instance_of(7).instance_id == (2, 0)


def test_cli_print_config_and_run(capsys):
    from psrl_b200.trainer.main import main
    assert main(["--preset", "cpu_tiny_grpo", "--print-config", "psrl.staleness=2"]) == 0
    out = capsys.readouterr().out
    assert "staleness: 2" in out
    assert main(["--preset", "cpu_tiny_grpo", "--steps", "1", "rollout.max_response_length=8"]) == 0
    assert '"step": 0' in capsys.readouterr().out


def test_native_router_core_prefix_and_policies():
    import random

    import numpy as np

    from psrl_b200.native import router
    _router = router()
    ix = _router.PrefixIndex(4, 3)
    ix.insert(np.arange(8))                    # 2 blocks
    assert ix.match(np.arange(12)) == 8 and ix.match(np.array([9, 9, 9, 9])) == 0
    ix.insert(np.arange(100, 108))             # 2 more blocks: capacity 3 evicts the oldest
    assert len(ix) == 3 and ix.match(np.arange(8)) == 0
    rng = random.Random(0)
    for _ in range(200):
        n = rng.randint(1, 6)
        load = [rng.randint(0, 40) for _ in range(n)]
        kv = [rng.random() for _ in range(n)]
        match = [rng.choice([0, 16, 32]) for _ in range(n)]
        # request_num_balance: first minimal (load, kv)
        assert _router.pick("request_num_balance", load, kv, match, 0, 1024, 16, 1.5, 7271.5, 0.05, 1.0) == \
            min(range(n), key=lambda i: (load[i], kv[i]))
        # cache_aware without imbalance: longest match, then least loaded
        i = _router.pick("cache_aware", load, kv, match, 0, 1024, 10 ** 6, 1.5, 7271.5, 0.05, 1.0)
        assert i == max(range(n), key=lambda j: (match[j], -load[j], -j))
        # throughput_optimal: the concave curve's marginal gain is largest at the lowest load
        t = _router.pick("throughput_optimal", load, kv, match, 0, 1024, 16, 1.5, 7271.5, 0.05, 1.0)
        assert load[t] == min(load)
