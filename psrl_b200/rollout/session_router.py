"""Session router: a session-scoped, OpenAI-style completion API for external
agents (C22).

External (black-box) agents talk HTTP; each session pins the weight version
of its first turn (later turns keep it so the trajectory's staleness is that
of its oldest tokens), sticks to one rollout instance (prefix-KV reuse), and
can be *hung* / *continued* by the scheduler.  Every turn is recorded as a
TITO record so the finished session becomes a training sample.

Routes (FastAPI):

* ``POST /v1/sessions/{sid}/completions`` ``{"prompt_ids": [...], "max_tokens": n}``
* ``POST /v1/sessions/{sid}/close`` → the TITO training sample
* ``POST /control/hang`` / ``POST /control/continue`` ``{"session_ids": [...]}``
* ``GET  /sessions`` — session states

Reference: ``psrl/workers/gen/session_router.py:36-360``.
"""

from __future__ import annotations

import itertools
import threading
from dataclasses import asdict, dataclass, field

from ..agent.tito import TurnRecord, build_training_data


@dataclass
class SessionState:
    session_id: str
    version_tag: int = -1
    instance_id: tuple | None = None
    hung: bool = False
    status: str = "env"          # gen (a turn is generating) | env (between turns)
    pending_obs_tokens: int = 0  # expected observation tokens of the next turn
    turns: list = field(default_factory=list)

    def context_tokens(self) -> int:
        return len(self.turns[-1].input_ids) + len(self.turns[-1].output_ids) if self.turns else 0


class SessionRouter:
    """``generate_fn(prompt_ids, max_tokens, version_tag, instance_hint) ->
    (output_ids, logprobs, versions, version_tag, instance_id)``."""

    def __init__(self, generate_fn, scheduler=None):
        """``scheduler`` (``session_scheduler.ThunderAgentScheduler``): after
        every turn boundary the sessions' KV footprints are checked against its
        capacity and sessions are hung (their next turn refused with 409 until
        continued) or continued."""
        self.generate = generate_fn
        self.scheduler = scheduler
        self.sessions: dict[str, SessionState] = {}
        self.lock = threading.Lock()
        self.sched_stats = {"hung": 0, "continued": 0}

    def _schedule(self) -> None:
        """Run the capacity scheduler over every open session (lock held)."""
        if self.scheduler is None:
            return
        from .session_scheduler import SessionInfo
        infos = [SessionInfo(k, v.context_tokens(), "hung" if v.hung else v.status, v.pending_obs_tokens)
                 for k, v in self.sessions.items()]
        to_hang, to_cont = self.scheduler.decide(infos)
        for k in to_hang:
            self.sessions[k].hung = True
        for k in to_cont:
            self.sessions[k].hung = False
        self.sched_stats["hung"] += len(to_hang)
        self.sched_stats["continued"] += len(to_cont)

    def complete(self, sid: str, prompt_ids: list[int], max_tokens: int) -> dict:
        with self.lock:
            s = self.sessions.setdefault(sid, SessionState(sid))
            if s.hung:
                return {"error": "session is hung", "status": 409}
            prev = s.context_tokens()
            s.pending_obs_tokens = max(0, len(prompt_ids) - prev)
            s.status = "gen"
            self._schedule()
        out, lps, vers, tag, inst = self.generate(prompt_ids, max_tokens, s.version_tag, s.instance_id)
        with self.lock:
            if s.version_tag < 0:
                s.version_tag = tag
            s.instance_id = inst
            s.turns.append(TurnRecord(list(prompt_ids), list(out), list(lps), list(vers)))
            s.status = "env"                      # the environment acts before the next turn
            self._schedule()
        return {"session_id": sid, "output_ids": out, "logprobs": lps, "version_tag": s.version_tag}

    def close(self, sid: str) -> dict:
        with self.lock:
            s = self.sessions.pop(sid)
            self._schedule()                      # freed capacity may continue hung sessions
        smp = build_training_data(s.turns)
        return {"session_id": sid, "version_tag": s.version_tag, **asdict(smp)}

    def hang(self, ids) -> list[str]:
        with self.lock:
            for i in ids:
                if i in self.sessions:
                    self.sessions[i].hung = True
            return [i for i in ids if i in self.sessions]

    def cont(self, ids) -> list[str]:
        with self.lock:
            for i in ids:
                if i in self.sessions:
                    self.sessions[i].hung = False
            return [i for i in ids if i in self.sessions]

    def states(self) -> dict:
        with self.lock:
            return {k: {"version_tag": v.version_tag, "hung": v.hung, "turns": len(v.turns),
                        "context_tokens": v.context_tokens()} for k, v in self.sessions.items()}

    def app(self):
        from fastapi import Body, FastAPI, HTTPException

        api = FastAPI(title="psrl_b200 session router")

        @api.post("/v1/sessions/{sid}/completions")
        def completions(sid: str, body: dict = Body(...)):
            r = self.complete(sid, list(body["prompt_ids"]), int(body.get("max_tokens", 64)))
            if "error" in r:
                raise HTTPException(status_code=r["status"], detail=r["error"])
            return r

        @api.post("/v1/sessions/{sid}/close")
        def close(sid: str):
            if sid not in self.sessions:
                raise HTTPException(404, "unknown session")
            return self.close(sid)

        @api.post("/control/hang")
        def control_hang(body: dict = Body(...)):
            return {"hung": self.hang(body.get("session_ids", []))}

        @api.post("/control/continue")
        def control_continue(body: dict = Body(...)):
            return {"continued": self.cont(body.get("session_ids", []))}

        @api.get("/sessions")
        def sessions():
            return self.states()

        return api


def engine_generate_fn(engines: list, temperature: float = 1.0):
    """A ``generate_fn`` for :class:`SessionRouter` over this framework's
    rollout engines: a session sticks to the engine that served its first
    turn (its KV prefix stays there), new sessions go round-robin, and each
    request carries the session's pinned version tag (the engine's current
    weight version for a first turn).  One lock per engine; the calling
    thread steps the engine until its request finishes."""
    from .engine import GenRequest, SamplingParams
    locks = [threading.Lock() for _ in engines]
    rr = itertools.count()
    ids = itertools.count(1 << 41)

    def generate(prompt_ids, max_tokens, version_tag, instance_hint):
        k = int(instance_hint[0]) if instance_hint is not None else next(rr) % len(engines)
        eng = engines[k]
        rid = next(ids)
        with locks[k]:
            tag = int(version_tag) if version_tag is not None and version_tag >= 0 else int(eng.version)
            params = SamplingParams(temperature=temperature, max_tokens=int(max_tokens), seed=rid & 0xFFFFF)
            eng.add_request(GenRequest(rid, list(prompt_ids), params, tag, {}))
            while True:
                for o in eng.step():
                    if o.request_id == rid:
                        return list(o.output_ids), list(o.logprobs), list(o.versions), tag, (k, 0)
                if not eng.has_unfinished():
                    raise RuntimeError("engine dropped the session request")

    return generate


class LocalSessionClient:
    """In-process client of one session (what an external agent would do
    over HTTP): ``complete(prompt_ids, max_tokens)`` returns the output ids,
    ``close()`` the session's TITO training sample."""

    def __init__(self, router: SessionRouter, sid: str):
        self.router = router
        self.sid = sid

    def complete(self, prompt_ids: list[int], max_tokens: int, wait_s: float = 600.0) -> list[int]:
        """A hung session waits (polling, at most ``wait_s``) until the
        scheduler continues it, as an HTTP client retrying on 409 would."""
        import time
        t0 = time.monotonic()
        while True:
            r = self.router.complete(self.sid, list(prompt_ids), int(max_tokens))
            if r.get("status") != 409:
                break
            if time.monotonic() - t0 > wait_s:
                raise TimeoutError(f"session {self.sid} stayed hung for {wait_s} s")
            time.sleep(0.005)
        if "error" in r:
            raise RuntimeError(r["error"])
        return list(r["output_ids"])

    def close(self) -> dict:
        return self.router.close(self.sid)
