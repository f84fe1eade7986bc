"""Reward functions and the reward-loop registry.

Registered loops (reference ``psrl/workers/reward/reward_loop/registry.py:22``):

* ``naive`` — score = task reward;
* ``dapo`` — task reward plus the DAPO overlong-buffer penalty
  ``-min(1, (len - (max_len - buffer)) / buffer) * factor`` beyond the soft limit;
* ``bernoulli_hash`` — Bernoulli(p) decided by a seeded hash of the trajectory id
  (synthetic benchmark reward);
* ``addition`` — 1.0 if the integer after the ``####`` marker equals the sum;
* ``prime``, ``gdpo``, ``gen`` — process-pool scoring with timeouts,
  multi-component rewards and the generative reward model (``loops.py``).

``RewardManager.score`` is called per finished trajectory on the driver;
``normalize_reward`` mirrors the reference's batch normalisation hook.
"""

from __future__ import annotations

import hashlib
import re
from typing import Callable

from . import loops as _loops

REWARD_LOOPS: dict[str, Callable] = {}


def register_reward_loop(name: str):
    def deco(fn):
        REWARD_LOOPS[name] = fn
        return fn
    return deco


def bernoulli_hash_score(traj_id: int, p: float, seed: int = 0) -> float:
    h = hashlib.blake2b(f"{seed}:{traj_id}".encode(), digest_size=8).digest()
    u = int.from_bytes(h, "little") / 2**64
    return 1.0 if u < p else 0.0


_NUM = re.compile(r"####\s*(-?\d+)")


def addition_score(response_text: str, answer: int) -> float:
    m = _NUM.search(response_text)
    return 1.0 if (m is not None and int(m.group(1)) == answer) else 0.0


def overlong_penalty(resp_len: int, max_len: int, buffer_len: int, factor: float) -> float:
    soft = max_len - buffer_len
    if resp_len <= soft or buffer_len <= 0:
        return 0.0
    return -min(1.0, (resp_len - soft) / buffer_len) * factor


@register_reward_loop("bernoulli_hash")
def _bernoulli(ctx, traj) -> dict:
    return {"score": bernoulli_hash_score(traj.request_id, ctx["p"], ctx.get("seed", 0))}


@register_reward_loop("addition")
def _addition(ctx, traj) -> dict:
    text = ctx["tokenizer"].decode(traj.response_ids)
    return {"score": addition_score(text, traj.meta.get("answer", -1))}


@register_reward_loop("naive")
def _naive(ctx, traj) -> dict:
    base = REWARD_LOOPS[ctx.get("task", "bernoulli_hash")]
    return base(ctx, traj)


@register_reward_loop("dapo")
def _dapo(ctx, traj) -> dict:
    base = REWARD_LOOPS[ctx.get("task", "bernoulli_hash")](ctx, traj)
    ob = ctx.get("overlong_buffer")
    pen = 0.0
    if ob and ob.get("enable"):
        pen = overlong_penalty(traj.response_len, ctx["max_response_length"], int(ob["len"]),
                               float(ob["penalty_factor"]))
    return {"score": base["score"] + pen, "acc": base["score"], "overlong_penalty": pen}


@register_reward_loop("env")
def _env(ctx, traj) -> dict:
    """The reward the episode's environment reported (e.g. the shell task's tests)."""
    info = (traj.meta or {}).get("env_info") or {}
    return {"score": float(info.get("reward", 0.0)), **{k: float(v) for k, v in info.items()
                                                        if isinstance(v, (int, float)) and k != "reward"}}


register_reward_loop("prime")(_loops.prime_loop)
register_reward_loop("gdpo")(_loops.gdpo_loop)
register_reward_loop("gen")(_loops.gen_loop)


def _cuda_available() -> bool:
    import torch
    return torch.cuda.is_available()


class RewardManager:
    """``reward_model``: the service the ``gen`` loop sends judge prompts to
    (anything with ``generate(prompt_ids) -> str``); built from
    ``reward.gen_rm`` when it names the ``http`` backend."""

    def __init__(self, cfg, tokenizer=None, reward_model=None):
        r = cfg.reward
        self.kind = r.kind
        self.ctx = {
            "p": float(r.get("p", 0.3)),
            "seed": int(cfg.data.get("seed", 0)),
            "tokenizer": tokenizer,
            "overlong_buffer": r.get("overlong_buffer"),
            "max_response_length": int(cfg.rollout.max_response_length),
            "task": r.get("task", "bernoulli_hash" if r.kind in ("naive", "dapo") else r.kind),
            "num_processes": int(r.get("num_processes", 8)),
            "timeout_s": float(r.get("timeout_s", 300.0)),
            "gdpo_components": list(r.get("gdpo_components") or []),
        }
        cs = r.get("compute_score")
        if cs:
            from ..utils.common import load_object
            self.ctx["compute_score"] = load_object(cs)
        else:
            self.ctx["compute_score"] = _loops.default_compute_score
        g = r.get("gen_rm") or {}
        self.ctx["gen_rm_function"] = g.get("function", "default")
        if reward_model is None and self.kind == "gen":
            if g.get("backend") == "http" and g.get("url"):
                reward_model = _loops.HttpRewardModel(g["url"], tokenizer, int(g.get("max_tokens", 512)),
                                                      float(g.get("temperature", 0.0)), model=g.get("model"))
            elif g.get("backend", "engine") == "engine" and (g.get("preset") or g.get("path")):
                dev = "cuda" if cfg.trainer.get("device", "auto") != "cpu" and _cuda_available() else "cpu"
                reward_model = _loops.build_engine_reward_model(g, tokenizer, dev)
        self.ctx["reward_model"] = reward_model
        if ":" in self.kind:
            # user code named in the config: "package.module:fn" or "path/file.py:fn",
            # called as fn(ctx, traj) -> {"score": float, ...}
            from ..utils.common import load_object
            self._fn = load_object(self.kind)
        elif self.kind not in REWARD_LOOPS:
            raise KeyError(f"unknown reward loop {self.kind!r}; registered: {sorted(REWARD_LOOPS)}")
        else:
            self._fn = REWARD_LOOPS[self.kind]

    def score(self, traj) -> dict:
        return self._fn(self.ctx, traj)

    def close(self) -> None:
        scorer = self.ctx.pop("_prime", None)
        if scorer is not None:
            scorer.close()

    @staticmethod
    def normalize_reward(scores: list[float]) -> list[float]:
        if len(scores) < 2:
            return list(scores)
        m = sum(scores) / len(scores)
        sd = (sum((s - m) ** 2 for s in scores) / (len(scores) - 1)) ** 0.5
        return [(s - m) / (sd + 1e-6) for s in scores]
