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

import threading
from dataclasses import asdict, dataclass, field

from ..agent.tito import TurnRecord, build_training_data


@dataclass
class SessionState:
    session_id: str
    version_tag: int = -1
    instance_id: tuple | None = None
    hung: bool = False
    turns: list = field(default_factory=list)

    def context_tokens(self) -> int:
        return len(self.turns[-1].input_ids) + len(self.turns[-1].output_ids) if self.turns else 0


class SessionRouter:
    """``generate_fn(prompt_ids, max_tokens, version_tag, instance_hint) ->
    (output_ids, logprobs, versions, version_tag, instance_id)``."""

    def __init__(self, generate_fn):
        self.generate = generate_fn
        self.sessions: dict[str, SessionState] = {}
        self.lock = threading.Lock()

    def complete(self, sid: str, prompt_ids: list[int], max_tokens: int) -> dict:
        with self.lock:
            s = self.sessions.setdefault(sid, SessionState(sid))
            if s.hung:
                return {"error": "session is hung", "status": 409}
        out, lps, vers, tag, inst = self.generate(prompt_ids, max_tokens, s.version_tag, s.instance_id)
        with self.lock:
            if s.version_tag < 0:
                s.version_tag = tag
            s.instance_id = inst
            s.turns.append(TurnRecord(list(prompt_ids), list(out), list(lps), list(vers)))
        return {"session_id": sid, "output_ids": out, "logprobs": lps, "version_tag": s.version_tag}

    def close(self, sid: str) -> dict:
        with self.lock:
            s = self.sessions.pop(sid)
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
