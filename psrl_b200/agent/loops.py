"""Agent loops (C13): how one trajectory is produced from one request.

* ``GenerateAgentLoop`` — single turn (the default; the engine's output is the
  trajectory).
* ``MultiTurnAgentLoop`` — alternates model turns and environment steps: after
  each turn the environment returns an observation, the context grows by
  (turn output + observation) and the next turn is resubmitted with a sticky
  hint so the rollout engine reuses the cached prefix KV; when the environment
  ends the episode the TITO builder assembles the sample (env tokens masked).
* ``SessionAgentLoop`` — the agent drives: a user agent function runs per
  task against a session of the session router (the same calls an external
  agent makes over its HTTP API), and the closed session's TITO record is
  the sample (reference ``loops/session_agent_loop.py``).

The registry mirrors the reference's Hydra-registered loop names
(``psrl/workers/agent_loop/loops/``).
"""

from __future__ import annotations

import threading

import numpy as np

from ..rollout.engine import GenRequest, RequestOutput, SamplingParams
from .envs import Environment, SyntheticTokenEnv
from .tito import TurnRecord, build_training_data

AGENT_LOOPS: dict = {}


def register_agent_loop(name):
    def deco(cls):
        AGENT_LOOPS[name] = cls
        return cls
    return deco


@register_agent_loop("single_turn")
class GenerateAgentLoop:
    multi_turn = False

    def on_turn_complete(self, o: RequestOutput, instance_id=None):
        return None

    def finalize(self, o: RequestOutput) -> dict:
        return {"prompt_ids": list(o.prompt_ids), "response_ids": list(o.output_ids), "logprobs": list(o.logprobs),
                "versions": list(o.versions), "response_mask": None, "turns": 1}


@register_agent_loop("multi_turn")
class MultiTurnAgentLoop:
    multi_turn = True

    def __init__(self, env_factory, turn_len_fn, max_turns: int = 8, ignore_eos: bool = True):
        self.env_factory = env_factory
        self.ignore_eos = bool(ignore_eos)
        self.turn_len = turn_len_fn
        self.max_turns = max_turns
        self.sessions: dict[int, dict] = {}
        self.lock = threading.Lock()

    def _session(self, o: RequestOutput) -> dict:
        s = self.sessions.get(o.request_id)
        if s is None:
            env: Environment = self.env_factory()
            env.reset({**o.meta, "uid": o.meta.get("uid", 0), "request_id": o.request_id})
            s = {"env": env, "turns": [], "tag": o.version_tag, "info": {}}
            self.sessions[o.request_id] = s
        return s

    def on_turn_complete(self, o: RequestOutput, instance_id=None) -> GenRequest | None:
        """Returns the next turn's request, or None when the episode ended."""
        with self.lock:
            s = self._session(o)
            s["turns"].append(TurnRecord(list(o.prompt_ids), list(o.output_ids), list(o.logprobs), list(o.versions)))
            turn = len(s["turns"]) - 1
            obs, done, info = s["env"].step(turn, list(o.output_ids))
            s["info"] = dict(info or {})
            if done or turn + 1 >= self.max_turns:
                return None
            ctx = list(o.prompt_ids) + list(o.output_ids) + list(obs)
            meta = dict(o.meta)
            meta["turn"] = turn + 1
            if instance_id is not None:
                meta["sticky_instance"] = tuple(instance_id)
            mt = int(self.turn_len(o.request_id, turn + 1))
            meta["max_tokens"] = mt
            params = SamplingParams(max_tokens=mt, ignore_eos=self.ignore_eos, seed=o.request_id * 7919 + 17 + turn + 1)
            return GenRequest(o.request_id, ctx, params, s["tag"], meta)

    def finalize(self, o: RequestOutput) -> dict:
        with self.lock:
            s = self.sessions.pop(o.request_id, None)
        if s:
            s["env"].close()
        turns = s["turns"] if s else [TurnRecord(list(o.prompt_ids), list(o.output_ids), list(o.logprobs),
                                                 list(o.versions))]
        smp = build_training_data(turns)
        return {"prompt_ids": smp.prompt_ids, "response_ids": smp.response_ids, "logprobs": smp.rollout_logprobs,
                "versions": smp.versions, "response_mask": smp.response_mask, "turns": smp.turn_count,
                "env_info": s["info"] if s else {}}

    def drop(self, request_id: int) -> None:
        with self.lock:
            s = self.sessions.pop(request_id, None)
        if s:
            s["env"].close()


@register_agent_loop("session")
class SessionAgentLoop:
    """Runs ``agent_fn(client, task)`` for each task on ``workers`` threads;
    ``client.complete(prompt_ids, max_tokens)`` goes through ``router`` (a
    :class:`SessionRouter`, e.g. over :func:`engine_generate_fn`).  Returns
    one sample per task: the TITO fields plus ``version_tag`` and the task,
    or ``error`` when the agent raised (its session is closed either way)."""

    multi_turn = True

    def __init__(self, router, agent_fn, workers: int = 8):
        self.router = router
        self.agent_fn = agent_fn
        self.workers = max(1, int(workers))

    def run(self, tasks: list[dict]) -> list[dict]:
        from concurrent.futures import ThreadPoolExecutor

        from ..rollout.session_router import LocalSessionClient

        def one(i_task):
            i, task = i_task
            sid = str(task.get("session_id", f"task-{i}"))
            client = LocalSessionClient(self.router, sid)
            err = None
            try:
                self.agent_fn(client, task)
            except Exception as exc:       # the agent's failure ends its episode only
                err = f"{type(exc).__name__}: {exc}"
            if sid not in self.router.sessions:
                return {"task": task, "error": err or "agent made no request"}
            smp = client.close()
            smp["task"] = task
            if err:
                smp["error"] = err
            return smp

        with ThreadPoolExecutor(self.workers, thread_name_prefix="session-agent") as ex:
            return list(ex.map(one, enumerate(tasks)))

    @staticmethod
    def to_trajectories(samples: list[dict], uid: int, request_id_base: int = 0) -> list:
        """Trajectories of one prompt group (``uid``) from finished session
        samples (failed sessions are skipped); ``reward`` is taken from the
        task's ``reward`` field when the agent left one there."""
        from ..trainer.batch import Trajectory
        out = []
        for j, smp in enumerate(samples):
            if "response_ids" not in smp or smp.get("error"):
                continue
            task = smp.get("task") or {}
            out.append(Trajectory(uid=uid, request_id=request_id_base + j, prompt_ids=list(smp["prompt_ids"]),
                                  response_ids=list(smp["response_ids"]),
                                  rollout_logprobs=list(smp["rollout_logprobs"]), reward=float(task.get("reward", 0.0)),
                                  versions=list(smp.get("versions") or []), version_tag=int(smp["version_tag"]),
                                  response_mask=list(smp["response_mask"]),
                                  meta={k: v for k, v in task.items() if k != "reward"}))
        return out


def build_agent_loop(cfg, vocab_size: int, tokenizer=None):
    """``psrl.agentic_rl.env`` picks the environment of multi-turn episodes:
    ``synthetic_tokens`` (the benchmark workload), ``shell_env`` or
    ``tool_env`` (decoded turns; ``rollout.max_response_length`` tokens per
    turn, stopping at EOS)."""
    turns = int(cfg.psrl.agentic_rl.get("max_turns", 1))
    if turns <= 1:
        return GenerateAgentLoop()
    ar = cfg.psrl.agentic_rl
    env_name = str(ar.get("env", "synthetic_tokens"))
    if env_name != "synthetic_tokens":
        from .envs import make_environment
        kw = {"tokenizer": tokenizer, "max_turns": turns}
        if env_name == "shell_env":
            kw.update(timeout_s=float(ar.get("command_timeout_s", 30.0)), docker_image=ar.get("docker_image"))
        elif env_name == "tool_env":
            from .tools import ToolRegistry
            kw.update(tools=ToolRegistry(), parser=str(ar.get("tool_parser", "hermes")))
        per_turn = int(cfg.rollout.max_response_length)
        return MultiTurnAgentLoop(lambda: make_environment(env_name, **kw), lambda rid, turn: per_turn, turns,
                                  ignore_eos=False)
    d = cfg.data
    mu, sigma, cap = float(d.response_len_mu), float(d.response_len_sigma), int(d.response_len_cap)
    ar = cfg.psrl.agentic_rl
    lo, hi = int(ar.get("obs_len_min", 128)), int(ar.get("obs_len_max", 1024))
    seed = int(d.seed)

    def turn_len(rid, turn):
        rng = np.random.default_rng([seed, rid, turn, 7])
        return int(min(cap, max(1, rng.lognormal(mu, sigma))))

    return MultiTurnAgentLoop(lambda: SyntheticTokenEnv(vocab_size, turns, lo, hi, seed), turn_len, turns)
