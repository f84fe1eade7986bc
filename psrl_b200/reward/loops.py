"""Reward loops beyond the task scorers: verifiable-answer scoring, PRIME's
process-pool scoring with timeouts, GDPO's multi-component rewards, and the
generative reward model (an LLM judge) with its serving backends.

* ``default_compute_score(data_source, solution_str, ground_truth,
  extra_info)`` — the scorer the loops use unless ``reward.compute_score``
  names one (``"package.module:fn"`` with the same signature, returning a
  float or a dict with ``score``).  ``####``-marked integers for arithmetic
  data, the last ``\\boxed{...}`` for math, exact match otherwise.
* ``prime`` — each score runs in a worker process (``reward.num_processes``)
  with a per-sample timeout (``reward.timeout_s``); a timeout or an
  exception scores 0 and is counted.  Reference:
  ``psrl/workers/reward/reward_loop/prime.py``.
* ``gdpo`` — the scorer returns a dict of reward components; ``score`` is
  their sum and ``components`` (in ``reward.gdpo_components`` order, or
  sorted keys) feeds the GDPO estimator, which normalises each component
  within its group.  Reference: ``psrl/workers/reward/reward_loop/gdpo.py``.
* ``gen`` — a generative reward model judges the response: a registered
  judge function (``reward.gen_rm.function``) builds the chat prompt from
  the decoded problem and solution, a reward-model service generates the
  critique, and the judge parses the score (``\\boxed{True}`` = 1 for the
  default judge).  Services: ``engine`` (replicas of this framework's
  rollout engine serving the reward model's weights, round-robin) and
  ``http`` (an OpenAI-style ``/v1/completions`` endpoint through the
  bounded POST pool).  Reference: ``psrl/workers/reward/reward_loop/gen.py``,
  ``gen_reward_function/``, ``reward_model/``.
"""

from __future__ import annotations

import itertools
import re
import threading
from multiprocessing import TimeoutError as mp_TimeoutError
from typing import Callable

# ------------------------------------------------------------------ scoring

_HASH_ANS = re.compile(r"####\s*(-?[\d,\.]+)")


def last_boxed(text: str) -> str | None:
    """Content of the last ``\\boxed{...}`` (balanced braces), or None."""
    i = text.rfind("\\boxed")
    if i < 0:
        return None
    j = text.find("{", i)
    if j < 0:
        return None
    depth = 0
    for k in range(j, len(text)):
        c = text[k]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return text[j + 1:k]
    return None


def _norm(s) -> str:
    s = str(s).strip().replace(" ", "").replace(",", "").rstrip(".")
    if s.startswith("\\text{") and s.endswith("}"):
        s = s[6:-1]
    try:
        f = float(s)
        return str(int(f)) if f == int(f) else repr(f)
    except ValueError:
        return s


def default_compute_score(data_source, solution_str: str, ground_truth, extra_info=None):
    """1.0 when the response's final answer equals ``ground_truth``."""
    ds = str(data_source or "")
    if ds in ("addition", "gsm8k") or "####" in solution_str:
        m = _HASH_ANS.findall(solution_str)
        return 1.0 if m and _norm(m[-1]) == _norm(ground_truth) else 0.0
    boxed = last_boxed(solution_str)
    if boxed is not None:
        return 1.0 if _norm(boxed) == _norm(ground_truth) else 0.0
    return 1.0 if _norm(solution_str) == _norm(ground_truth) else 0.0


def _as_result(res) -> dict:
    if isinstance(res, dict):
        out = dict(res)
        out["score"] = float(out.get("score", 0.0))
        return out
    return {"score": float(res)}


def _inputs(ctx, traj) -> tuple:
    tok = ctx["tokenizer"]
    meta = traj.meta or {}
    gt = meta.get("ground_truth", meta.get("answer"))
    src = meta.get("data_source", ctx.get("task"))
    text = tok.decode([i for i, m in zip(traj.response_ids, traj.response_mask or [1] * traj.response_len) if m])
    return src, text, gt, {k: v for k, v in meta.items() if k not in ("ground_truth", "data_source")}


# ------------------------------------------------------------------- prime


class ProcessScorer:
    """Scores in worker processes with a per-sample timeout (the scorer must
    be importable by name, i.e. a module-level function).  A timed-out
    scorer may never return, so its pool is terminated and replaced: a stuck
    worker neither blocks later samples nor the process's exit."""

    def __init__(self, fn: Callable, num_processes: int, timeout_s: float):
        self.fn = fn
        self.timeout = float(timeout_s)
        self.n = max(1, int(num_processes))
        self.stats = {"timeouts": 0, "errors": 0}
        self.lock = threading.Lock()
        self.pool = self._new_pool()

    def _new_pool(self):
        # spawned workers: the scoring process is multi-threaded (fork would copy held locks)
        import multiprocessing as mp
        return mp.get_context("spawn").Pool(self.n)

    def __call__(self, *args) -> dict:
        with self.lock:
            pool = self.pool
        res = pool.apply_async(self.fn, args)
        try:
            return _as_result(res.get(timeout=self.timeout))
        except mp_TimeoutError:
            with self.lock:
                self.stats["timeouts"] += 1
                if self.pool is pool:
                    pool.terminate()
                    self.pool = self._new_pool()
            return {"score": 0.0, "timeout": 1.0}
        except Exception:       # a failing scorer scores 0, as a timeout does
            with self.lock:
                self.stats["errors"] += 1
            return {"score": 0.0, "error": 1.0}

    def close(self) -> None:
        with self.lock:
            self.pool.terminate()
            self.pool.join()


def prime_loop(ctx, traj) -> dict:
    scorer = ctx.get("_prime")
    if scorer is None:
        scorer = ctx["_prime"] = ProcessScorer(ctx["compute_score"], ctx.get("num_processes", 8),
                                               ctx.get("timeout_s", 300.0))
    return scorer(*_inputs(ctx, traj))


# -------------------------------------------------------------------- gdpo


def gdpo_loop(ctx, traj) -> dict:
    res = ctx["compute_score"](*_inputs(ctx, traj))
    if not isinstance(res, dict):
        res = {"score": float(res)}
    names = ctx.get("gdpo_components") or sorted(k for k, v in res.items()
                                                 if k != "score" and isinstance(v, (int, float)))
    if not names:
        names = ["score"]
    comps = [float(res.get(k, 0.0)) for k in names]
    out = {k: float(v) for k, v in res.items() if isinstance(v, (int, float))}
    out["score"] = float(sum(comps)) if names != ["score"] else float(res["score"])
    out["components"] = comps
    return out


# --------------------------------------------------- generative reward model

GEN_RM_FUNCTIONS: dict[str, type] = {}


def gen_reward_function(name: str):
    def deco(cls):
        GEN_RM_FUNCTIONS[name] = cls
        return cls
    return deco


@gen_reward_function("default")
class BoxedVerdictJudge:
    """Asks the reward model to critique a solution and put ``True`` or
    ``False`` in ``\\boxed{}``; the score is 1.0 for ``True``."""

    template = ("Below is a problem and a candidate solution.\n\n[Problem]\n{problem}\n\n[Solution]\n{solution}\n\n"
                "Check the solution step by step and decide whether it is correct. "
                "Give the verdict (True or False) inside \\boxed{{}}.")

    def prompt(self, problem: str, solution: str) -> list[dict]:
        return [{"role": "user", "content": self.template.format(problem=problem, solution=solution)}]

    def score(self, rm_output: str, **_) -> float:
        v = last_boxed(rm_output)
        return 1.0 if v is not None and v.strip() == "True" else 0.0


@gen_reward_function("scalar")
class ScalarJudge:
    """Asks for a 0-10 rating in ``\\boxed{}``; the score is rating / 10."""

    template = ("Rate the response to the prompt from 0 (useless) to 10 (perfect).\n\n[Prompt]\n{problem}\n\n"
                "[Response]\n{solution}\n\nPut the rating inside \\boxed{{}}.")

    def prompt(self, problem: str, solution: str) -> list[dict]:
        return [{"role": "user", "content": self.template.format(problem=problem, solution=solution)}]

    def score(self, rm_output: str, **_) -> float:
        v = last_boxed(rm_output)
        try:
            return min(1.0, max(0.0, float(v) / 10.0)) if v is not None else 0.0
        except ValueError:
            return 0.0


class EngineRewardModel:
    """Reward-model replicas served by the framework's own rollout engine
    (one lock per replica; requests go round-robin).  ``generate`` returns
    the decoded completion of one prompt."""

    def __init__(self, engines: list, tokenizer, max_tokens: int = 512, temperature: float = 0.0):
        self.engines = list(engines)
        self.locks = [threading.Lock() for _ in self.engines]
        self.tok = tokenizer
        self.max_tokens = int(max_tokens)
        self.temperature = float(temperature)
        self._rr = itertools.count()
        self._ids = itertools.count(1 << 40)

    def generate(self, prompt_ids: list[int]) -> str:
        from ..rollout.engine import GenRequest, SamplingParams
        k = next(self._rr) % len(self.engines)
        eng = self.engines[k]
        rid = next(self._ids)
        params = SamplingParams(temperature=self.temperature, max_tokens=self.max_tokens, seed=rid & 0xFFFF)
        with self.locks[k]:
            eng.add_request(GenRequest(rid, list(prompt_ids), params))
            while True:
                for o in eng.step():
                    if o.request_id == rid:
                        return self.tok.decode(o.output_ids)
                if not eng.has_unfinished():
                    raise RuntimeError("reward-model engine dropped the request")


def build_engine_reward_model(gcfg, tokenizer, device: str = "cpu") -> EngineRewardModel:
    """Reward-model replicas from ``reward.gen_rm``: the model named by
    ``preset`` or ``path`` (an HF directory; weights loaded when present),
    ``replicas`` engines on ``device``, each with ``kv_cache_gb`` of KV."""
    import torch

    from ..models import build_model, model_args_from_config
    from ..models.hf_io import load_hf_into
    from ..rollout.engine import EngineWeights, RolloutEngine
    args = model_args_from_config({"preset": gcfg.get("preset"), "path": gcfg.get("path")})
    dev = torch.device(gcfg.get("device") or device)
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    engines = []
    for _ in range(max(1, int(gcfg.get("replicas", 1)))):
        m = build_model(args, dev, dtype, seed=int(gcfg.get("seed", 0)))
        if gcfg.get("path"):
            load_hf_into(m, gcfg["path"])
        engines.append(RolloutEngine(args, EngineWeights.from_model(m, dev, dtype),
                                     max_num_seqs=int(gcfg.get("max_num_seqs", 16)),
                                     max_model_len=int(gcfg.get("max_model_len", 4096)), block_size=16,
                                     kv_cache_gb=float(gcfg.get("kv_cache_gb", 1.0)),
                                     use_cuda_graph=dev.type == "cuda"))
        del m
    return EngineRewardModel(engines, tokenizer, int(gcfg.get("max_tokens", 512)), float(gcfg.get("temperature", 0.0)))


class HttpRewardModel:
    """An OpenAI-style completions endpoint (``POST {url}/v1/completions``,
    answer in ``choices[0].text``) through the bounded POST pool."""

    def __init__(self, url: str, tokenizer, max_tokens: int = 512, temperature: float = 0.0, pool=None,
                 model: str | None = None):
        from ..utils.common import HttpPostPool
        self.url = url.rstrip("/") + "/v1/completions"
        self.tok = tokenizer
        self.max_tokens = int(max_tokens)
        self.temperature = float(temperature)
        self.model = model
        self.pool = pool or HttpPostPool()

    def generate(self, prompt_ids: list[int]) -> str:
        payload = {"prompt": self.tok.decode(prompt_ids), "max_tokens": self.max_tokens,
                   "temperature": self.temperature}
        if self.model:
            payload["model"] = self.model
        res = self.pool.submit(self.url, payload).result()
        return str(res["choices"][0]["text"])


def gen_loop(ctx, traj) -> dict:
    from ..utils.common import apply_chat_template
    rm = ctx.get("reward_model")
    if rm is None:
        raise RuntimeError("reward.kind=gen needs a reward-model service (RewardManager(reward_model=...) "
                           "or reward.gen_rm.backend=http with reward.gen_rm.url)")
    judge = ctx.get("_judge")
    if judge is None:
        judge = ctx["_judge"] = GEN_RM_FUNCTIONS[ctx.get("gen_rm_function", "default")]()
    tok = ctx["tokenizer"]
    _, solution, gt, _ = _inputs(ctx, traj)
    problem = tok.decode(traj.prompt_ids)
    ids = apply_chat_template(judge.prompt(problem, solution), tok)
    out = rm.generate(ids)
    return {"score": float(judge.score(out, ground_truth=gt)), "rm_output_len": float(len(out))}
