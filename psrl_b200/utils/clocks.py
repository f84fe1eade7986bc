"""Sample GPU SM clocks and throttle reasons with ``nvidia-smi`` while a timed
region runs (read-only queries; nothing about the GPU is changed)."""

from __future__ import annotations

import statistics
import subprocess

FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
          "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
          "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


class ClockSampler:
    def __init__(self, gpu_indices: list[int] | None = None, interval_ms: int = 200):
        self.gpus = gpu_indices
        self.interval_ms = interval_ms
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={','.join(FIELDS)}", "--format=csv,noheader,nounits",
               f"-lms={self.interval_ms}"]
        if self.gpus is not None:
            cmd.append("-i=" + ",".join(str(g) for g in self.gpus))
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        return summarize([ln for ln in out.splitlines() if ln.strip()])


def summarize(lines: list[str]) -> dict:
    sm, smax, power = [], [], []
    reasons: set[str] = set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for ln in lines:
        parts = [p.strip() for p in ln.split(",")]
        if len(parts) < len(FIELDS):
            continue
        try:
            sm.append(float(parts[1]))
            smax.append(float(parts[2]))
            power.append(float(parts[3]))
        except ValueError:
            continue
        for nm, val in zip(names, parts[5:9]):
            if val.lower() == "active":
                reasons.add(nm)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "power_w_max": max(power),
            "reasons": sorted(reasons), "samples": len(sm)}
