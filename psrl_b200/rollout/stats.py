"""Engine statistics: snapshots, JSONL recorder, ZMQ push/pull transport (C25).

``EngineStats`` is the per-instance load snapshot the router and coordinator
consume (queue lengths, generation throughput, KV utilisation).  Snapshots can
be recorded to JSONL and shipped between processes over ZMQ PUSH/PULL
(reference ``psrl/workers/gen/stats_collector.py``, ``stats_recorder.py``,
``zmq_queue.py``).
"""

from __future__ import annotations

import json
import os
import time
from dataclasses import asdict, dataclass, field


@dataclass
class EngineStats:
    instance_id: tuple = (0, 0)
    version: int = 0
    num_waiting: int = 0
    num_running: int = 0
    kv_usage: float = 0.0
    gen_throughput: float = 0.0       # tokens/s over the last window
    prefix_hit_rate: float = 0.0
    num_preemptions: int = 0
    ts: float = field(default_factory=time.time)

    @classmethod
    def from_engine(cls, instance_id, engine, window: "ThroughputWindow | None" = None) -> "EngineStats":
        st = engine.engine_stats()
        return cls(tuple(instance_id), st["version"], st["num_waiting"], st["num_running"], st["kv_usage"],
                   window.rate(st["decode_tokens"]) if window else 0.0, st["prefix_hit_rate"], st["preemptions"])

    def to_dict(self) -> dict:
        return asdict(self)


class ThroughputWindow:
    def __init__(self):
        self.t = time.monotonic()
        self.n = 0

    def rate(self, total_tokens: int) -> float:
        now = time.monotonic()
        dt = max(1e-6, now - self.t)
        r = (total_tokens - self.n) / dt
        self.t, self.n = now, total_tokens
        return r


class StatsRecorder:
    def __init__(self, path: str):
        self.path = os.path.expanduser(path)
        os.makedirs(os.path.dirname(self.path) or ".", exist_ok=True)

    def record(self, stats: EngineStats | dict) -> None:
        d = stats.to_dict() if isinstance(stats, EngineStats) else dict(stats)
        with open(self.path, "a") as fh:
            fh.write(json.dumps(d, default=str) + "\n")

    def read(self) -> list[dict]:
        if not os.path.exists(self.path):
            return []
        with open(self.path) as fh:
            return [json.loads(ln) for ln in fh if ln.strip()]


class ZMQPushQueue:
    def __init__(self, address: str):
        import zmq
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.PUSH)
        self.sock.connect(address)

    def put(self, obj) -> None:
        self.sock.send_pyobj(obj)

    def close(self):
        self.sock.close(0)


class ZMQPullQueue:
    def __init__(self, address: str):
        import zmq
        self.zmq = zmq
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.PULL)
        self.sock.bind(address)

    def get(self, timeout_ms: int = 1000):
        if self.sock.poll(timeout_ms):
            return self.sock.recv_pyobj()
        return None

    def close(self):
        self.sock.close(0)
