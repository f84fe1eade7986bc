"""Rollout router: PSRL worker selection (C21 / N1, the SMG router's role).

Selection pipeline for one request over the live instances:

1. **version filter** — only instances whose weight version is at least the
   request's version tag (a partial rollout never moves back in version);
2. **sticky hint** — a partial/sticky request prefers the instance that holds
   its KV (trajectory stickiness), a group member prefers its siblings'
   instance (group stickiness);
3. **admission** — the PS must accept the request at the instance's version
   (``can_reserve_request`` / ``get_reserve_indicator``);
4. **policy** — ``random``, ``round_robin``, ``request_num_balance`` (fewest
   running + waiting), ``throughput_optimal`` (largest marginal throughput from
   the instance's fitted throughput curve, optionally within a request budget)
   or ``cache_aware`` (longest prefix match in the instance's recent-prefix
   index, unless the load imbalance exceeds the balance thresholds).

The prefix index and the policy arithmetic run in the native router core
(``csrc_host/router_core.cpp``, module ``psrl_b200._router``); the stages that
consult Python objects (eligibility, PS admission, stickiness) stay here.

Reference: ``psrl/workers/gen/smg_adapter.py:47-153`` (router arguments) and
``docs/design/router_tito.md``.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field

import numpy as np


@dataclass
class InstanceState:
    instance_id: tuple
    version: int = 0
    num_running: int = 0
    num_waiting: int = 0
    kv_usage: float = 0.0
    throughput: float = 0.0
    healthy: bool = True
    paused: bool = False
    max_concurrent: int = 1024
    meta: dict = field(default_factory=dict)

    @property
    def load(self) -> int:
        return self.num_running + self.num_waiting


class PrefixIndex:
    """Per-instance LRU set of block-hash chains of recently routed prompts
    (native: ``csrc_host/router_core.cpp``)."""

    def __init__(self, block_size: int = 16, max_entries: int = 1 << 16):
        from ..native import router as _native_router
        _router = _native_router()
        self.bs = block_size
        self._ix = _router.PrefixIndex(block_size, max_entries)

    def match(self, tokens) -> int:
        return int(self._ix.match(np.asarray(tokens, dtype=np.int64)))

    def insert(self, tokens) -> None:
        self._ix.insert(np.asarray(tokens, dtype=np.int64))

    def __len__(self) -> int:
        return len(self._ix)


class ThroughputModel:
    """tokens/s ~= A * (1 - (B * x + 1) ** -k) for x concurrent requests
    (the curve the reference fits per model, ``trainer/config/throughput_model``)."""

    def __init__(self, A: float = 7271.5, B: float = 0.05, k: float = 1.0):
        self.A, self.B, self.k = A, B, k

    def rate(self, x: float) -> float:
        return self.A * (1.0 - (self.B * x + 1.0) ** (-self.k))

    def marginal(self, x: float) -> float:
        return self.rate(x + 1) - self.rate(x)


class Router:
    POLICIES = ("random", "round_robin", "request_num_balance", "throughput_optimal",
                "throughput_optimal_with_budget", "cache_aware", "cache_aware_v1")

    def __init__(self, method: str = "request_num_balance", ps=None, *, group_sticky: bool = False,
                 trajectory_sticky: bool = True, request_budget: int = 1024, block_size: int = 16,
                 balance_abs_threshold: int = 16, balance_rel_threshold: float = 1.5, seed: int = 0,
                 throughput_model: ThroughputModel | None = None):
        if method not in self.POLICIES:
            raise ValueError(f"unknown routing policy {method!r}")
        self.method = method
        self.ps = ps
        self.group_sticky = group_sticky
        self.trajectory_sticky = trajectory_sticky
        self.request_budget = request_budget
        self.balance_abs = balance_abs_threshold
        self.balance_rel = balance_rel_threshold
        self.rng = random.Random(seed)
        self.rr = 0
        self.prefix: dict[tuple, PrefixIndex] = {}
        self.group_home: dict[int, tuple] = {}
        self.tput = throughput_model or ThroughputModel()
        self.block_size = block_size

    # -------------------------------------------------------------- stages
    def eligible(self, req, instances: list[InstanceState]) -> list[InstanceState]:
        tag = max(-1, int(getattr(req, "version_tag", -1)))
        return [s for s in instances if s.healthy and not s.paused and s.version >= tag and s.load < s.max_concurrent]

    def admit(self, req, cands: list[InstanceState]) -> list[InstanceState]:
        if self.ps is None:
            return cands
        out = []
        for s in cands:
            ind = self.ps.get_reserve_indicator(req.request_id, [s.version])[0]
            if ind != float("inf"):
                out.append((ind, s))
        # prefer instances where the group already has a reservation (-inf), then any
        out.sort(key=lambda x: x[0])
        return [s for _, s in out]

    def sticky(self, req, cands: list[InstanceState]) -> InstanceState | None:
        ids = {s.instance_id: s for s in cands}
        hint = req.meta.get("sticky_instance") if self.trajectory_sticky else None
        if hint is not None and tuple(hint) in ids:
            return ids[tuple(hint)]
        if self.group_sticky:
            home = self.group_home.get(req.meta.get("uid"))
            if home in ids:
                return ids[home]
        return None

    # -------------------------------------------------------------- policy
    def pick(self, req, cands: list[InstanceState]) -> InstanceState:
        """Policy choice among admitted candidates (native core except ``random``)."""
        from ..native import router as _native_router
        _router = _native_router()
        m = self.method
        if m == "random":
            return self.rng.choice(cands)
        loads = [s.load for s in cands]
        kv = [float(s.kv_usage) for s in cands]
        match = [0] * len(cands)
        if m.startswith("cache_aware"):
            toks = list(req.prompt_ids) + list(getattr(req, "prev_output_ids", []))
            match = [self.prefix.setdefault(s.instance_id, PrefixIndex(self.block_size)).match(toks) for s in cands]
        i = _router.pick(m, loads, kv, match, self.rr, self.request_budget, self.balance_abs, float(self.balance_rel),
                         float(self.tput.A), float(self.tput.B), float(self.tput.k))
        if m == "round_robin":
            self.rr += 1
        return cands[i]

    def route(self, req, instances: list[InstanceState]) -> InstanceState | None:
        cands = self.eligible(req, instances)
        if not cands:
            return None
        s = self.sticky(req, cands)
        if s is None:
            cands = self.admit(req, cands)
            if not cands:
                return None
            s = self.pick(req, cands)
        s.num_waiting += 1
        self.group_home.setdefault(req.meta.get("uid"), s.instance_id)
        if self.method.startswith("cache_aware"):
            self.prefix.setdefault(s.instance_id, PrefixIndex(self.block_size)).insert(
                list(req.prompt_ids) + list(getattr(req, "prev_output_ids", [])))
        return s

    @classmethod
    def from_cfg(cls, cfg, ps=None) -> "Router":
        """Router of ``psrl.rollout_coordination.routing_strategy``."""
        rs = cfg.psrl.rollout_coordination.routing_strategy
        cap = rs.get("cache_aware_policy", {}) or {}
        return cls(str(rs.method), ps, group_sticky=bool(rs.get("enable_group_sticky", False)),
                   trajectory_sticky=bool(rs.get("enable_trajectory_sticky", False)),
                   request_budget=int(rs.get("request_budget", 1024)), block_size=int(rs.get("block_size", 16)),
                   balance_abs_threshold=int(cap.get("balance_abs_threshold", 16)),
                   balance_rel_threshold=float(cap.get("balance_rel_threshold", 1.5)))

    def assigned(self, req, s: InstanceState) -> None:
        """Record that ``req`` went to ``s`` (pull mode): group home, the
        instance's prefix index, its queued count."""
        s.num_waiting += 1
        self.group_home.setdefault(req.meta.get("uid"), s.instance_id)
        if self.method.startswith("cache_aware"):
            self.prefix.setdefault(s.instance_id, PrefixIndex(self.block_size)).insert(
                list(req.prompt_ids) + list(getattr(req, "prev_output_ids", [])))

    def accepts(self, req, me: InstanceState, instances: list[InstanceState]) -> bool:
        """Pull-mode check: should instance ``me`` take ``req`` now?"""
        s = self.sticky(req, self.eligible(req, instances))
        if s is not None:
            return s.instance_id == me.instance_id
        if self.method in ("random", "round_robin"):
            return True
        best = self.pick(req, self.eligible(req, instances) or [me])
        return best.instance_id == me.instance_id or best.load >= me.load
