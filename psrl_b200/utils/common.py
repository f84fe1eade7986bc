"""Common helpers (C39): dynamic import of user code named in a config, worker
naming, compact serialisation of samples, a ChatML chat template, a bounded
HTTP POST pool for external services (reward models, sandboxes,
environments), and a safety-net cleanup of labelled Docker containers.

Reference: ``psrl/utils/common/*.py`` (``worker_naming.py``, ``http_utils.py``,
dynamic import and serialisation helpers, chat templates).
"""

from __future__ import annotations

import importlib
import importlib.util
import json
import os
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any

# ------------------------------------------------------------ dynamic import


def load_object(spec: str) -> Any:
    """``"package.module:attr"`` or ``"/path/file.py:attr"`` -> the attribute.
    Lets a config name a custom reward function, agent loop or tool."""
    if ":" not in spec:
        raise ValueError(f"expected 'module:attr' or 'file.py:attr', got {spec!r}")
    mod_name, attr = spec.rsplit(":", 1)
    if mod_name.endswith(".py") or os.sep in mod_name:
        path = os.path.abspath(mod_name)
        name = "psrl_user_" + os.path.splitext(os.path.basename(path))[0]
        sp = importlib.util.spec_from_file_location(name, path)
        if sp is None or sp.loader is None:
            raise ImportError(f"cannot load {path}")
        mod = importlib.util.module_from_spec(sp)
        sp.loader.exec_module(mod)
    else:
        mod = importlib.import_module(mod_name)
    obj = mod
    for part in attr.split("."):
        obj = getattr(obj, part)
    return obj


# ------------------------------------------------------------- worker names


def worker_name(role: str, rank: int, instance: tuple | int | None = None) -> str:
    """Stable, parseable process / endpoint names: ``trainer-r3``,
    ``rollout-i2.0-r5`` (instance id (2, 0) on rank 5)."""
    if instance is None:
        return f"{role}-r{int(rank)}"
    inst = ".".join(str(int(x)) for x in instance) if isinstance(instance, (tuple, list)) else str(int(instance))
    return f"{role}-i{inst}-r{int(rank)}"


def parse_worker_name(name: str) -> dict:
    parts = name.split("-")
    out: dict = {"role": parts[0]}
    for p in parts[1:]:
        if p.startswith("r"):
            out["rank"] = int(p[1:])
        elif p.startswith("i"):
            out["instance"] = tuple(int(x) for x in p[1:].split("."))
    return out


# ------------------------------------------------------------ serialisation


def pack_sample(sample: dict) -> bytes:
    """Compact bytes for a sample dict of token lists / floats / strings
    (msgpack; lists of ints and floats stay lists)."""
    import msgpack
    return msgpack.packb(sample, use_bin_type=True)


def unpack_sample(data: bytes) -> dict:
    import msgpack
    return msgpack.unpackb(data, raw=False, strict_map_key=False)


# ------------------------------------------------------------ chat template


def chatml(messages: list[dict], add_generation_prompt: bool = True) -> str:
    """Qwen-style ChatML: ``<|im_start|>{role}\\n{content}<|im_end|>\\n`` per
    message, then ``<|im_start|>assistant\\n`` when a reply is to follow.
    Tool results use the ``tool`` role as Qwen2.5 does."""
    out = []
    for m in messages:
        role = m.get("role", "user")
        content = m.get("content", "")
        if not isinstance(content, str):
            content = json.dumps(content, ensure_ascii=False)
        out.append(f"<|im_start|>{role}\n{content}<|im_end|>\n")
    if add_generation_prompt:
        out.append("<|im_start|>assistant\n")
    return "".join(out)


def apply_chat_template(messages: list[dict], tokenizer, add_generation_prompt: bool = True) -> list[int]:
    """Token ids of the ChatML rendering (uses the tokenizer's own template
    when it has one, e.g. an HF tokenizer)."""
    if hasattr(tokenizer, "apply_chat_template"):
        return list(tokenizer.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                                  tokenize=True))
    return list(tokenizer.encode(chatml(messages, add_generation_prompt)))


# ------------------------------------------------------------- HTTP pool


class HttpPostPool:
    """Bounded pool of JSON POSTs with per-call timeout and retries.

    ``submit(url, payload)`` returns a Future of the decoded JSON response;
    at most ``max_inflight`` requests run at once (the reference's POST actor
    pool).  The transport is injectable (``post(url, json, timeout) -> dict``)
    so the pool is testable without a network.
    """

    def __init__(self, max_inflight: int = 64, timeout_s: float = 60.0, retries: int = 2, backoff_s: float = 0.5,
                 post=None):
        self.timeout = float(timeout_s)
        self.retries = int(retries)
        self.backoff = float(backoff_s)
        self._post = post or self._requests_post
        self._ex = ThreadPoolExecutor(max_workers=max_inflight, thread_name_prefix="http-post")
        self._lock = threading.Lock()
        self.stats = {"ok": 0, "retried": 0, "failed": 0}

    @staticmethod
    def _requests_post(url: str, payload: dict, timeout: float) -> dict:
        import requests
        r = requests.post(url, json=payload, timeout=timeout)
        r.raise_for_status()
        return r.json()

    def _call(self, url: str, payload: dict) -> dict:
        last: Exception | None = None
        for attempt in range(self.retries + 1):
            try:
                res = self._post(url, payload, self.timeout)
                with self._lock:
                    self.stats["ok"] += 1
                return res
            except Exception as exc:      # network / HTTP errors: retry with backoff
                last = exc
                if attempt < self.retries:
                    with self._lock:
                        self.stats["retried"] += 1
                    time.sleep(self.backoff * (2 ** attempt))
        with self._lock:
            self.stats["failed"] += 1
        raise RuntimeError(f"POST {url} failed after {self.retries + 1} attempts: {last}") from last

    def submit(self, url: str, payload: dict) -> Future:
        return self._ex.submit(self._call, url, payload)

    def close(self) -> None:
        self._ex.shutdown(wait=True)


# ------------------------------------------------------------------ docker


def remove_containers_by_label(label: str = "psrl=episode", run=None) -> int:
    """Force-remove every Docker container carrying ``label`` (episode
    containers a crashed worker left behind).  Returns how many were
    removed; 0 when Docker is not installed.  ``run`` replaces
    ``subprocess.run`` (tests)."""
    import shutil
    import subprocess
    run = run or subprocess.run
    if run is subprocess.run and shutil.which("docker") is None:
        return 0
    ps = run(["docker", "ps", "-aq", "--filter", f"label={label}"], capture_output=True, text=True, timeout=60)
    ids = [x for x in (ps.stdout or "").split() if x]
    if ids:
        run(["docker", "rm", "-f", *ids], capture_output=True, text=True, timeout=120)
    return len(ids)
