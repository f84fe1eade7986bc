"""The elastic executor driving engines through EngineFleet (CPU: fake
engines with the engine's sleep / wake interface): low load puts the least
loaded instance to sleep and hands its interrupted requests back, high load
wakes it, level-2 sleeps reload weights after waking."""

import types

from psrl_b200.utils.elastic import EngineFleet, ScalingPolicy


class FakeEngine:
    def __init__(self, running):
        self.asleep = False
        self.running = list(range(running))
        self.waiting = []
        self.stats = {"decode_tokens": 0}
        self.bm = types.SimpleNamespace(usage=lambda: 0.2)
        self.slept = self.woken = 0

    def sleep(self, keep_weights=True):
        self.asleep = True
        self.slept += 1
        outs = [("abort", r) for r in self.running]
        self.running = []
        return outs, 1 << 30

    def wake(self):
        self.asleep = False
        self.woken += 1
        return 1 << 30


def test_executor_sleeps_idle_engine_and_wakes_it_under_load():
    a, b = FakeEngine(running=5), FakeEngine(running=1)
    back = []
    fleet = EngineFleet({(0, 0): a, (1, 0): b}, on_interrupted=back.extend)
    pol = ScalingPolicy(cooldown_ms=0, min_awake=1)
    ex = fleet.executor(pol)
    pol.observe_arrivals(0, 1.0)                # nothing arriving: scale down
    d = ex.tick()
    assert d.action == "down" and d.instance_id == (1, 0)
    assert b.asleep and b.slept == 1 and back == [("abort", 0)]
    assert fleet.released_bytes == 1 << 30
    for _ in range(5):                          # a burst of arrivals: scale up
        pol.observe_arrivals(10_000, 1.0)
    d = ex.tick()
    assert d.action == "up" and d.instance_id == (1, 0) and not b.asleep and b.woken == 1
    assert [h.action for h in ex.history] == ["down", "up"]


def test_level2_sleep_reloads_weights_after_wake():
    e = FakeEngine(running=0)
    reloaded = []
    fleet = EngineFleet({(0, 0): e}, keep_weights=False, reload=lambda iid, eng: reloaded.append(iid))
    fleet.sleep((0, 0))
    fleet.wake((0, 0))
    assert reloaded == [(0, 0)]
