"""Begin/end event logging with durations (C32).

Event types follow the reference's ``EventType`` (``psrl/utils/logger/ray_logger.py:28``):
PULL, PUSH, BUFFER_READY, INIT, TRAIN, GEN, VAL, WAIT, SWITCH, OTHER.  Events are
kept in memory and optionally appended as JSON lines; the timeline viewer
(:mod:`psrl_b200.utils.visualize`) renders them.
"""

from __future__ import annotations

import contextlib
import json
import os
import threading
import time
from enum import Enum


class EventType(str, Enum):
    PULL = "PULL"
    PUSH = "PUSH"
    BUFFER_READY = "BUFFER_READY"
    INIT = "INIT"
    TRAIN = "TRAIN"
    GEN = "GEN"
    VAL = "VAL"
    WAIT = "WAIT"
    SWITCH = "SWITCH"
    OTHER = "OTHER"


class EventLog:
    def __init__(self, path: str | None = None, actor: str = "driver", keep: int = 100_000):
        self.path = os.path.expanduser(path) if path else None
        self.actor = actor
        self.events: list[dict] = []
        self.keep = keep
        self._lock = threading.Lock()
        if self.path:
            os.makedirs(os.path.dirname(self.path) or ".", exist_ok=True)

    def emit(self, name: str, kind: str | EventType = EventType.OTHER, **fields) -> dict:
        ev = {"ts": time.time(), "actor": self.actor, "name": name, "type": str(EventType(kind).value), **fields}
        with self._lock:
            self.events.append(ev)
            if len(self.events) > self.keep:
                del self.events[: len(self.events) - self.keep]
            if self.path:
                with open(self.path, "a") as fh:
                    fh.write(json.dumps(ev, default=str) + "\n")
        return ev

    @contextlib.contextmanager
    def span(self, kind: str | EventType, name: str | None = None, **fields):
        t0 = time.time()
        self.emit(name or str(kind), kind, phase="begin", **fields)
        try:
            yield
        finally:
            self.emit(name or str(kind), kind, phase="end", duration_s=time.time() - t0, **fields)

    def record_span(self, kind: str | EventType, start_ts: float, duration_s: float, name: str | None = None,
                    **fields) -> None:
        """A span measured elsewhere (``start_ts`` wall-clock seconds): its
        begin and end events, in the same form as :meth:`span` writes."""
        k = str(EventType(kind).value)
        for ev in ({"ts": start_ts, "phase": "begin"},
                   {"ts": start_ts + duration_s, "phase": "end", "duration_s": duration_s}):
            ev.update({"actor": self.actor, "name": name or k, "type": k, **fields})
            with self._lock:
                self.events.append(ev)
                if len(self.events) > self.keep:
                    del self.events[: len(self.events) - self.keep]
                if self.path:
                    with open(self.path, "a") as fh:
                        fh.write(json.dumps(ev) + "\n")

    def durations(self, kind: str) -> list[float]:
        return [e["duration_s"] for e in self.events if e["type"] == kind and e.get("phase") == "end"]


def rank_event_log(cfg, rank: int, role: str) -> EventLog:
    """The event log of one rank: ``trainer.event_log_dir/events_rank{rank}.jsonl``
    when that directory is set, in memory only otherwise."""
    d = cfg.trainer.get("event_log_dir", None) if cfg is not None else None
    path = None
    if d:
        os.makedirs(os.path.expanduser(str(d)), exist_ok=True)
        path = os.path.join(str(d), f"events_rank{rank}.jsonl")
    return EventLog(path, actor=f"{role}{rank}")
