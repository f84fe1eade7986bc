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
