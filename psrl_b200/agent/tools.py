"""Tools for agent loops (C24): ``BaseTool``, ``FunctionTool`` and HTTP-backed
tools (SandboxFusion code execution, MCP servers).  Remote tools need their
endpoint configured; they are rate-limited with :class:`TokenBucket`."""

from __future__ import annotations

import inspect
import json
from typing import Callable

from ..utils.concurrency import TokenBucket


class BaseTool:
    name = "tool"
    description = ""
    parameters: dict = {}

    def schema(self) -> dict:
        return {"type": "function", "function": {"name": self.name, "description": self.description,
                                                 "parameters": self.parameters}}

    def execute(self, arguments: dict) -> str:
        raise NotImplementedError


class FunctionTool(BaseTool):
    def __init__(self, fn: Callable, name: str | None = None, description: str = ""):
        self.fn = fn
        self.name = name or fn.__name__
        self.description = description or (fn.__doc__ or "").strip()
        sig = inspect.signature(fn)
        self.parameters = {"type": "object", "properties": {p: {"type": "string"} for p in sig.parameters},
                           "required": [p for p, v in sig.parameters.items() if v.default is inspect._empty]}

    def execute(self, arguments: dict) -> str:
        try:
            out = self.fn(**arguments)
        except Exception as exc:
            return f"error: {type(exc).__name__}: {exc}"
        return out if isinstance(out, str) else json.dumps(out, default=str)


class SandboxFusionTool(BaseTool):
    """Runs code in a SandboxFusion-compatible HTTP service (``POST {url}/run_code``)."""

    name = "code_interpreter"
    description = "Execute code in a sandbox and return stdout/stderr."
    parameters = {"type": "object", "properties": {"code": {"type": "string"}, "language": {"type": "string"}},
                  "required": ["code"]}

    def __init__(self, url: str, timeout_s: float = 30.0, rate_per_s: float = 8.0):
        self.url = url.rstrip("/")
        self.timeout = timeout_s
        self.bucket = TokenBucket(rate_per_s, rate_per_s)

    def execute(self, arguments: dict) -> str:
        import requests
        self.bucket.acquire()
        r = requests.post(f"{self.url}/run_code", json={"code": arguments.get("code", ""),
                                                      "language": arguments.get("language", "python")},
                          timeout=self.timeout)
        r.raise_for_status()
        d = r.json()
        run = d.get("run_result", d)
        return (run.get("stdout", "") or "") + (run.get("stderr", "") or "")


class MCPClientManager:
    """Calls tools exposed by MCP servers over their HTTP JSON-RPC endpoint."""

    def __init__(self, servers: dict[str, str], timeout_s: float = 30.0):
        self.servers = dict(servers)
        self.timeout = timeout_s
        self._id = 0

    def call(self, server: str, tool: str, arguments: dict) -> str:
        import requests
        self._id += 1
        body = {"jsonrpc": "2.0", "id": self._id, "method": "tools/call",
                "params": {"name": tool, "arguments": arguments}}
        r = requests.post(self.servers[server], json=body, timeout=self.timeout)
        r.raise_for_status()
        res = r.json().get("result", {})
        parts = res.get("content", [])
        return "".join(p.get("text", "") for p in parts if isinstance(p, dict))


class ToolRegistry:
    def __init__(self, tools: list[BaseTool] | None = None):
        self.tools = {t.name: t for t in (tools or [])}

    def register(self, tool: BaseTool) -> None:
        self.tools[tool.name] = tool

    def run(self, name: str, arguments: dict) -> str:
        t = self.tools.get(name)
        if t is None:
            return f"error: unknown tool {name!r}"
        return t.execute(arguments)
