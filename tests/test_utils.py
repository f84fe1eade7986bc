import json

from psrl_b200.utils.events import EventLog, EventType
from psrl_b200.utils.profiling import MemoryLogger, TurnProfilingCollector, TurnRecord, marked_timer
from psrl_b200.utils.visualize import render, spans


def test_events_spans_and_timeline(tmp_path):
    log = EventLog(str(tmp_path / "ev.jsonl"), actor="trainer")
    with log.span(EventType.TRAIN, step=1):
        pass
    with log.span(EventType.PUSH, step=1):
        pass
    assert len(log.durations("TRAIN")) == 1
    evs = [json.loads(x) for x in open(tmp_path / "ev.jsonl")]
    sp = spans(evs)
    assert {s["type"] for s in sp} == {"TRAIN", "PUSH"}
    page = render(evs)
    assert "<svg" in page and "trainer" in page


def test_profiling_records(tmp_path):
    c = TurnProfilingCollector(str(tmp_path / "p.jsonl"))
    c.add(TurnRecord(1, 0, 100, 20, cached_tokens=0))
    c.add(TurnRecord(1, 1, 130, 10, cached_tokens=128))
    assert c.data[1].totals()["cache_hit_rate"] > 0.5
    assert c.flush() == 1
    t = {}
    with marked_timer("gen", t):
        pass
    assert "gen" in t
    m = MemoryLogger()
    with m.around("x"):
        pass
    assert len(m.records) == 2


def test_elastic_policy_up_down_and_cooldown():
    from psrl_b200.utils.elastic import ElasticExecutor, InstanceSignal, ScalingPolicy, ThroughputFit
    pol = ScalingPolicy(theta_low=0.2, theta_max=0.8, cooldown_ms=1000, fit=ThroughputFit(A=1000, B=0.1, k=1,
                                                                                           tokens_per_request=100))
    sig = [InstanceSignal((0, 0), True, num_running=8), InstanceSignal((1, 0), False)]
    pol._lambda = 100.0                                   # far above one instance's service rate
    d = pol.decide(sig, now_ms=0)
    assert d.action == "up" and d.instance_id == (1, 0)
    assert pol.decide(sig, now_ms=500).action == "none"   # cooldown
    sig = [InstanceSignal((0, 0), True, num_running=1), InstanceSignal((1, 0), True, num_running=0)]
    pol._lambda = 0.0
    d = pol.decide(sig, now_ms=5000)
    assert d.action == "down" and d.instance_id == (1, 0)
    woke, slept = [], []
    ex = ElasticExecutor(ScalingPolicy(cooldown_ms=0), lambda: [InstanceSignal((0, 0), True, kv_usage=0.99),
                                                                 InstanceSignal((1, 0), False)],
                         slept.append, woke.append)
    ex.tick()
    assert woke == [(1, 0)]


def test_common_helpers(tmp_path):
    from psrl_b200.utils.common import (HttpPostPool, chatml, load_object, pack_sample, parse_worker_name,
                                        unpack_sample, worker_name)
    f = tmp_path / "myreward.py"
    f.write_text("def score(ctx, traj):\n    return {'score': float(len(traj.response_ids))}\n")
    fn = load_object(f"{f}:score")
    assert load_object("os.path:join") is __import__("os").path.join
    from psrl_b200.trainer.batch import Trajectory
    t = Trajectory(uid=0, request_id=1, prompt_ids=[1], response_ids=[2, 3, 4], rollout_logprobs=[0.0] * 3)
    assert fn({}, t)["score"] == 3.0
    n = worker_name("rollout", 5, (2, 0))
    assert n == "rollout-i2.0-r5" and parse_worker_name(n) == {"role": "rollout", "instance": (2, 0), "rank": 5}
    s = {"ids": [1, 2, 3], "lp": [-0.5, -1.25], "meta": {"turns": 2}}
    assert unpack_sample(pack_sample(s)) == s
    assert chatml([{"role": "user", "content": "hi"}]) == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    calls = {"n": 0}

    def flaky(url, payload, timeout):
        calls["n"] += 1
        if calls["n"] == 1:
            raise ConnectionError("first try fails")
        return {"echo": payload["x"]}
    pool = HttpPostPool(max_inflight=2, retries=2, backoff_s=0.0, post=flaky)
    assert pool.submit("http://unused", {"x": 7}).result(timeout=5) == {"echo": 7}
    assert pool.stats["retried"] == 1 and pool.stats["ok"] == 1
    pool.close()


def test_reward_from_user_module(tmp_path):
    f = tmp_path / "rw.py"
    f.write_text("def fn(ctx, traj):\n    return {'score': 0.25}\n")
    from psrl_b200.config import load_config
    from psrl_b200.reward import RewardManager
    from psrl_b200.trainer.batch import Trajectory
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"reward.kind={f}:fn"])
    rm = RewardManager(cfg)
    t = Trajectory(uid=0, request_id=1, prompt_ids=[1], response_ids=[2], rollout_logprobs=[0.0])
    assert rm.score(t)["score"] == 0.25


def test_remove_containers_by_label_with_fake_docker():
    from types import SimpleNamespace

    from psrl_b200.utils.common import remove_containers_by_label
    calls = []

    def run(argv, **kw):
        calls.append(argv)
        return SimpleNamespace(stdout="abc123\ndef456\n" if argv[1] == "ps" else "", returncode=0)

    assert remove_containers_by_label("psrl=episode", run=run) == 2
    assert calls[0][:4] == ["docker", "ps", "-aq", "--filter"] and calls[0][4] == "label=psrl=episode"
    assert calls[1] == ["docker", "rm", "-f", "abc123", "def456"]


def test_config_validation_of_new_groups():
    import pytest

    from psrl_b200.config import ConfigError, load_config
    for bad in (["algorithm.use_kl_in_reward=true", "algorithm.kl_ctrl.type=pid"],
                ["algorithm.rollout_correction.rollout_rs=banana"],
                ["data.kind=parquet"],
                ["reward.kind=gen", "reward.gen_rm.backend=http"],
                ["psrl.agentic_rl.env=moon"]):
        with pytest.raises(ConfigError):
            load_config(preset="cpu_tiny_grpo", overrides=bad)
