"""Profiling and tracing (C33): per-turn rollout records, stage timers, GPU
memory logging and an optional torch-profiler window.

* ``TurnProfilingCollector`` — per request/turn timings (queue wait, prefill,
  decode, environment), cache hits, preemptions and partial resumes, written
  as JSONL (reference ``psrl/utils/profiling/{collector,records}.py``).
* ``marked_timer`` — accumulate wall time per stage name into a dict.
* ``MemoryLogger`` — snapshots of ``torch.cuda`` allocator statistics per stage
  (reference ``psrl/utils/logger/memory_logger.py``).
* ``ProfilerWindow`` — torch.profiler over the configured steps, for
  diagnostics only (numbers taken under a profiler are never reported).
"""

from __future__ import annotations

import contextlib
import json
import os
import time
from dataclasses import asdict, dataclass, field

import torch


@dataclass
class TurnRecord:
    request_id: int
    turn: int
    prompt_tokens: int
    output_tokens: int
    cached_tokens: int = 0
    queue_s: float = 0.0
    prefill_s: float = 0.0
    decode_s: float = 0.0
    env_s: float = 0.0
    preemptions: int = 0
    partial_resumes: int = 0
    version_tag: int = 0


@dataclass
class TrajectoryProfilingData:
    request_id: int
    turns: list = field(default_factory=list)

    def totals(self) -> dict:
        t = {"turns": len(self.turns), "output_tokens": 0, "cached_tokens": 0, "prompt_tokens": 0}
        for r in self.turns:
            t["output_tokens"] += r.output_tokens
            t["cached_tokens"] += r.cached_tokens
            t["prompt_tokens"] += r.prompt_tokens
        t["cache_hit_rate"] = t["cached_tokens"] / max(1, t["prompt_tokens"])
        return t


class TurnProfilingCollector:
    def __init__(self, path: str | None = None):
        self.path = os.path.expanduser(path) if path else None
        self.data: dict[int, TrajectoryProfilingData] = {}

    def add(self, rec: TurnRecord) -> None:
        self.data.setdefault(rec.request_id, TrajectoryProfilingData(rec.request_id)).turns.append(rec)

    def from_output(self, o, turn: int = 0, queue_s: float = 0.0) -> TurnRecord:
        rec = TurnRecord(o.request_id, turn, len(o.prompt_ids), len(o.output_ids), o.num_cached_tokens,
                         queue_s=queue_s, version_tag=o.version_tag)
        self.add(rec)
        return rec

    def flush(self) -> int:
        if not self.path:
            return 0
        os.makedirs(os.path.dirname(self.path) or ".", exist_ok=True)
        n = 0
        with open(self.path, "a") as fh:
            for d in self.data.values():
                fh.write(json.dumps({"request_id": d.request_id, "turns": [asdict(t) for t in d.turns],
                                     **d.totals()}) + "\n")
                n += 1
        self.data.clear()
        return n


@contextlib.contextmanager
def marked_timer(name: str, timing: dict):
    t0 = time.perf_counter()
    try:
        yield
    finally:
        timing[name] = timing.get(name, 0.0) + time.perf_counter() - t0


class MemoryLogger:
    def __init__(self, device=None):
        self.device = device
        self.records: list[dict] = []

    def snapshot(self, tag: str) -> dict:
        if not torch.cuda.is_available():
            rec = {"tag": tag, "allocated_gb": 0.0, "reserved_gb": 0.0, "max_allocated_gb": 0.0}
        else:
            d = self.device if self.device is not None else torch.cuda.current_device()
            rec = {"tag": tag,
                   "allocated_gb": torch.cuda.memory_allocated(d) / 2**30,
                   "reserved_gb": torch.cuda.memory_reserved(d) / 2**30,
                   "max_allocated_gb": torch.cuda.max_memory_allocated(d) / 2**30}
        rec["ts"] = time.time()
        self.records.append(rec)
        return rec

    @contextlib.contextmanager
    def around(self, tag: str):
        self.snapshot(tag + ":begin")
        yield
        self.snapshot(tag + ":end")


def gpu_memory_logger_decorator(tag: str, logger: MemoryLogger):
    def deco(fn):
        def wrapped(*a, **k):
            with logger.around(tag):
                return fn(*a, **k)
        return wrapped
    return deco


class ProfilerWindow:
    """Runs torch.profiler for the listed steps (diagnostics; results are traces, not benchmark numbers)."""

    def __init__(self, steps: list[int], out_dir: str):
        self.steps = set(int(s) for s in steps)
        self.out_dir = os.path.expanduser(out_dir)
        self.prof = None

    def start(self, step: int) -> None:
        if step in self.steps and self.prof is None:
            from torch.profiler import ProfilerActivity, profile
            acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
            self.prof = profile(activities=acts, record_shapes=False)
            self.prof.__enter__()

    def stop(self, step: int) -> str | None:
        if self.prof is None:
            return None
        self.prof.__exit__(None, None, None)
        os.makedirs(self.out_dir, exist_ok=True)
        path = os.path.join(self.out_dir, f"trace_step{step}.json")
        self.prof.export_chrome_trace(path)
        self.prof = None
        return path


class StepObserver:
    """What every trainer step records besides its own metrics: allocator
    statistics on CUDA (``memory/allocated_gb``, ``memory/reserved_gb``,
    ``memory/max_allocated_gb``) and, for the steps listed in
    ``trainer.profile_steps``, a torch-profiler trace under
    ``trainer.profile_dir/rank{r}`` (the reference's ``global_profiler.steps``)."""

    def __init__(self, cfg, device, rank: int = 0):
        steps = list(cfg.trainer.get("profile_steps", None) or [])
        out = os.path.join(str(cfg.trainer.get("profile_dir", "torch_traces")), f"rank{rank}")
        self.window = ProfilerWindow(steps, out) if steps else None
        dev = torch.device(device)
        self.mem = MemoryLogger(dev) if dev.type == "cuda" else None

    def begin(self, step: int) -> None:
        if self.window is not None:
            self.window.start(step)

    def end(self, step: int, metrics: dict) -> None:
        if self.window is not None:
            path = self.window.stop(step)
            if path:
                metrics["profile/trace"] = path
        if self.mem is not None:
            r = self.mem.snapshot(f"step{step}")
            metrics.update({"memory/allocated_gb": r["allocated_gb"], "memory/reserved_gb": r["reserved_gb"],
                            "memory/max_allocated_gb": r["max_allocated_gb"]})
