"""Capacity-based session scheduling ("ThunderAgent", C23).

Long agentic sessions alternate model turns and environment time.  When the
KV demand of the sessions that want to run exceeds capacity, sessions are
*hung* (their KV released, their next turn held back) and later *continued*:

* hang: sessions in environment status first (they are not generating), then
  the smallest footprints first, until the running footprint fits;
* continue: best-fit-decreasing — repeatedly continue the largest hung session
  that still fits the free capacity.

Footprint of a session = context tokens (+ ``env_token_weight`` x expected
observation tokens while in the environment) in KV blocks.
Reference: ``rollout_coordination/session/thunder_agent.py:39-200``.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class SessionInfo:
    session_id: str
    context_tokens: int
    status: str = "gen"          # gen | env | hung
    pending_obs_tokens: int = 0

    def footprint(self, env_weight: float) -> float:
        extra = env_weight * self.pending_obs_tokens if self.status == "env" else 0.0
        return self.context_tokens + extra


class ThunderAgentScheduler:
    def __init__(self, capacity_tokens: int, env_token_weight: float = 1.0, buffer_per_session: int = 100):
        self.capacity = int(capacity_tokens)
        self.w = float(env_token_weight)
        self.buffer = int(buffer_per_session)

    def _need(self, s: SessionInfo) -> float:
        return s.footprint(self.w) + self.buffer

    def decide(self, sessions: list[SessionInfo]) -> tuple[list[str], list[str]]:
        """Returns (to_hang, to_continue) session ids."""
        active = [s for s in sessions if s.status != "hung"]
        hung = [s for s in sessions if s.status == "hung"]
        used = sum(self._need(s) for s in active)
        to_hang: list[str] = []
        if used > self.capacity:
            order = sorted(active, key=lambda s: (s.status != "env", self._need(s)))
            for s in order:
                if used <= self.capacity:
                    break
                to_hang.append(s.session_id)
                used -= self._need(s)
            return to_hang, []
        free = self.capacity - used
        to_continue: list[str] = []
        for s in sorted(hung, key=self._need, reverse=True):
            need = self._need(s)
            if need <= free:
                to_continue.append(s.session_id)
                free -= need
        return [], to_continue


def scheduler_from_cfg(cfg, capacity_tokens: int):
    """The scheduler of ``psrl.rollout_coordination.session_strategy.thunder_agent``
    (None unless enabled), for a pool whose KV cache holds ``capacity_tokens``
    (the engines' blocks x block size)."""
    ta = cfg.psrl.rollout_coordination.session_strategy.thunder_agent
    if not bool(ta.get("enable", False)):
        return None
    return ThunderAgentScheduler(int(capacity_tokens), float(ta.get("env_token_weight", 1.0)),
                                 int(ta.get("buffer_per_session", 100)))
