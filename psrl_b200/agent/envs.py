"""Environments for multi-turn agent loops (C24).

An environment reacts to a generated turn with an observation (token ids) and
says whether the episode is over.

* ``SyntheticTokenEnv`` — the agentic benchmark workload: a fixed number of
  turns, each observation is uniform-random tokens of length U[lo, hi].
* ``ToolEnv`` — decodes the turn, parses tool calls, runs them and returns the
  tool results as the next observation; done when the model stops calling tools.
* ``ShellTaskEnv`` — a software-engineering task in a per-episode workspace
  (the role of the reference's mini-SWE environment): each turn's last
  fenced ``bash`` block runs in the workspace (a local process, or ``docker
  exec`` in a per-episode container when ``docker_image`` is set) and its
  exit code and output are the observation; the episode ends when the model
  submits (``submit_marker``) or runs out of turns, and the task's
  ``test_cmd`` then grades the workspace (``info["reward"]`` 1.0 on success).

Environments are registered by name (``register_environment``,
``make_environment``; reference ``psrl/environments/base.py``
``Environment.register``).
"""

from __future__ import annotations

import os
import re
import shutil
import subprocess
import tempfile
import uuid

import numpy as np

from .tool_parser import get_parser
from .tools import ToolRegistry


ENVIRONMENTS: dict[str, type] = {}


def register_environment(name: str):
    def deco(cls):
        ENVIRONMENTS[name] = cls
        return cls
    return deco


def make_environment(name: str, **kwargs):
    if name not in ENVIRONMENTS:
        raise KeyError(f"unknown environment {name!r}; registered: {sorted(ENVIRONMENTS)}")
    return ENVIRONMENTS[name](**kwargs)


class Environment:
    max_turns: int = 1

    def close(self) -> None:
        pass

    def reset(self, task: dict) -> None:
        pass

    def step(self, turn: int, action_ids: list[int]) -> tuple[list[int], bool, dict]:
        """(observation ids, done, info) after the model's turn ``turn``."""
        raise NotImplementedError


@register_environment("synthetic_tokens")
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


@register_environment("tool_env")
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


_BASH_BLOCK = re.compile(r"```(?:bash|sh)\s*\n(.*?)```", re.S)


@register_environment("shell_env")
class ShellTaskEnv(Environment):
    """Shell-command episodes in a per-episode workspace.

    ``reset(task)`` creates the workspace and writes ``task["files"]``
    (path -> text) into it; ``task["test_cmd"]`` grades it at the end.  A
    command runs with ``timeout_s``; its output is cut to ``max_obs_chars``.
    With ``docker_image`` the workspace is bind-mounted into a container that
    lives for the episode (``docker run -d`` at reset, ``docker rm -f`` at
    close); without it commands run as local processes of the current user
    in the workspace, with no isolation beyond the working directory, so the
    container backend is the one for untrusted model output."""

    def __init__(self, tokenizer, max_turns: int = 8, timeout_s: float = 30.0, max_obs_chars: int = 4000,
                 submit_marker: str = "COMPLETE_TASK_AND_SUBMIT", docker_image: str | None = None,
                 workdir_root: str | None = None):
        self.tok = tokenizer
        self.max_turns = int(max_turns)
        self.timeout = float(timeout_s)
        self.max_obs = int(max_obs_chars)
        self.marker = submit_marker
        self.image = docker_image
        self.root = workdir_root
        self.ws: str | None = None
        self.container: str | None = None
        self.task: dict = {}

    def reset(self, task: dict) -> None:
        self.close()
        self.task = dict(task)
        self.ws = tempfile.mkdtemp(prefix="psrl_ws_", dir=self.root)
        for rel, text in (task.get("files") or {}).items():
            path = os.path.join(self.ws, rel)
            os.makedirs(os.path.dirname(path), exist_ok=True)
            with open(path, "w") as fh:
                fh.write(text)
        if self.image:
            self.container = f"psrl-{uuid.uuid4().hex[:12]}"
            subprocess.run(["docker", "run", "-d", "--rm", "--label", "psrl=episode", "--name", self.container,
                            "-v", f"{self.ws}:/workspace", "-w", "/workspace", self.image, "sleep", "infinity"],
                           check=True, capture_output=True, timeout=120)

    def run(self, cmd: str) -> tuple[int, str]:
        """Run one command; on timeout its whole process group is killed
        (commands may start background children)."""
        import signal
        argv = (["docker", "exec", "-w", "/workspace", self.container, "bash", "-lc", cmd] if self.container
                else ["bash", "-c", cmd])
        p = subprocess.Popen(argv, cwd=None if self.container else self.ws, stdout=subprocess.PIPE,
                             stderr=subprocess.STDOUT, text=True, start_new_session=True)
        try:
            out, _ = p.communicate(timeout=self.timeout)
            code = p.returncode
        except subprocess.TimeoutExpired:
            try:
                os.killpg(p.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            out, _ = p.communicate()
            out, code = (out or "") + f"\n[timed out after {self.timeout:g} s]", 124
        if len(out) > self.max_obs:
            half = self.max_obs // 2
            out = out[:half] + "\n[... output truncated ...]\n" + out[-half:]
        return code, out

    def grade(self) -> float:
        cmd = self.task.get("test_cmd")
        if not cmd:
            return 0.0
        code, _ = self.run(cmd)
        return 1.0 if code == 0 else 0.0

    def step(self, turn, action_ids):
        text = self.tok.decode(action_ids)
        blocks = _BASH_BLOCK.findall(text)
        submitted = self.marker in text
        if submitted or not blocks or turn + 1 >= self.max_turns:
            info = {"reward": self.grade(), "submitted": float(submitted), "commands": float(turn + 1)}
            return [], True, info
        code, out = self.run(blocks[-1])
        obs = f"<returncode>{code}</returncode>\n<output>\n{out}</output>\n"
        return self.tok.encode(obs), False, {"returncode": code}

    def close(self) -> None:
        if self.container:
            subprocess.run(["docker", "rm", "-f", self.container], capture_output=True, timeout=60)
            self.container = None
        if self.ws:
            shutil.rmtree(self.ws, ignore_errors=True)
            self.ws = None
