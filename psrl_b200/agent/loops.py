"""Agent loops (C13): how one trajectory is produced from one request.

* ``GenerateAgentLoop`` — single turn (the default; the engine's output is the
  trajectory).
* ``MultiTurnAgentLoop`` — alternates model turns and environment steps: after
  each turn the environment returns an observation, the context grows by
  (turn output + observation) and the next turn is resubmitted with a sticky
  hint so the rollout engine reuses the cached prefix KV; when the environment
  ends the episode the TITO builder assembles the sample (env tokens masked).

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

    def __init__(self, env_factory, turn_len_fn, max_turns: int = 8):
        self.env_factory = env_factory
        self.turn_len = turn_len_fn
        self.max_turns = max_turns
        self.sessions: dict[int, dict] = {}
        self.lock = threading.Lock()

    def _session(self, o: RequestOutput) -> dict:
        s = self.sessions.get(o.request_id)
        if s is None:
            env: Environment = self.env_factory()
            env.reset({"uid": o.meta.get("uid", 0), "request_id": o.request_id})
            s = {"env": env, "turns": [], "tag": o.version_tag}
            self.sessions[o.request_id] = s
        return s

    def on_turn_complete(self, o: RequestOutput, instance_id=None) -> GenRequest | None:
        """Returns the next turn's request, or None when the episode ended."""
        with self.lock:
            s = self._session(o)
            s["turns"].append(TurnRecord(list(o.prompt_ids), list(o.output_ids), list(o.logprobs), list(o.versions)))
            turn = len(s["turns"]) - 1
            obs, done, _ = s["env"].step(turn, list(o.output_ids))
            if done or turn + 1 >= self.max_turns:
                return None
            ctx = list(o.prompt_ids) + list(o.output_ids) + list(obs)
            meta = dict(o.meta)
            meta["turn"] = turn + 1
            if instance_id is not None:
                meta["sticky_instance"] = tuple(instance_id)
            mt = int(self.turn_len(o.request_id, turn + 1))
            meta["max_tokens"] = mt
            params = SamplingParams(max_tokens=mt, ignore_eos=True, seed=o.request_id * 7919 + 17 + turn + 1)
            return GenRequest(o.request_id, ctx, params, s["tag"], meta)

    def finalize(self, o: RequestOutput) -> dict:
        with self.lock:
            s = self.sessions.pop(o.request_id, None)
        turns = s["turns"] if s else [TurnRecord(list(o.prompt_ids), list(o.output_ids), list(o.logprobs),
                                                 list(o.versions))]
        smp = build_training_data(turns)
        return {"prompt_ids": smp.prompt_ids, "response_ids": smp.response_ids, "logprobs": smp.rollout_logprobs,
                "versions": smp.versions, "response_mask": smp.response_mask, "turns": smp.turn_count}

    def drop(self, request_id: int) -> None:
        with self.lock:
            self.sessions.pop(request_id, None)


def build_agent_loop(cfg, vocab_size: int):
    turns = int(cfg.psrl.agentic_rl.get("max_turns", 1))
    if turns <= 1:
        return GenerateAgentLoop()
    d = cfg.data
    mu, sigma, cap = float(d.response_len_mu), float(d.response_len_sigma), int(d.response_len_cap)
    ar = cfg.psrl.agentic_rl
    lo, hi = int(ar.get("obs_len_min", 128)), int(ar.get("obs_len_max", 1024))
    seed = int(d.seed)

    def turn_len(rid, turn):
        rng = np.random.default_rng([seed, rid, turn, 7])
        return int(min(cap, max(1, rng.lognormal(mu, sigma))))

    return MultiTurnAgentLoop(lambda: SyntheticTokenEnv(vocab_size, turns, lo, hi, seed), turn_len, turns)
