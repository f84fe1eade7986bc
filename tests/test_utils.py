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
