"""Environments for multi-turn agent loops (C24).

An environment reacts to a generated turn with an observation (token ids) and
says whether the episode is over.

* ``SyntheticTokenEnv`` — the agentic benchmark workload: a fixed number of
  turns, each observation is uniform-random tokens of length U[lo, hi].
* ``ToolEnv`` — decodes the turn, parses tool calls, runs them and returns the
  tool results as the next observation; done when the model stops calling tools.
"""

from __future__ import annotations

import numpy as np

from .tool_parser import get_parser
from .tools import ToolRegistry


class Environment:
    max_turns: int = 1

    def reset(self, task: dict) -> None:
        pass

    def step(self, turn: int, action_ids: list[int]) -> tuple[list[int], bool, dict]:
        """(observation ids, done, info) after the model's turn ``turn``."""
        raise NotImplementedError


class SyntheticTokenEnv(Environment):
    def __init__(self, vocab_size: int, max_turns: int = 8, obs_lo: int = 128, obs_hi: int = 1024, seed: int = 0):
        self.vocab = vocab_size
        self.max_turns = max_turns
        self.lo, self.hi = obs_lo, obs_hi
        self.seed = seed
        self.key = 0

    def reset(self, task: dict) -> None:
        self.key = int(task.get("uid", 0)) * 1000 + int(task.get("request_id", 0))

    def step(self, turn, action_ids):
        if turn + 1 >= self.max_turns:
            return [], True, {}
        rng = np.random.default_rng([self.seed, self.key, turn])
        n = int(rng.integers(self.lo, self.hi + 1))
        return rng.integers(3, self.vocab, size=n).tolist(), False, {}


class ToolEnv(Environment):
    def __init__(self, tokenizer, tools: ToolRegistry, parser: str = "hermes", max_turns: int = 4):
        self.tok = tokenizer
        self.tools = tools
        self.parse = get_parser(parser)
        self.max_turns = max_turns

    def step(self, turn, action_ids):
        text = self.tok.decode(action_ids)
        calls, _ = self.parse(text)
        if not calls or turn + 1 >= self.max_turns:
            return [], True, {"num_calls": len(calls)}
        results = [f"<tool_response>{self.tools.run(c.name, c.arguments)}</tool_response>" for c in calls]
        return self.tok.encode("\n".join(results)), False, {"num_calls": len(calls)}
