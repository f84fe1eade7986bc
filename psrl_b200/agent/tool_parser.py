"""Tool-call parsers for model outputs (C24).

Each parser turns generated text into ``[ToolCall(name, arguments)]`` plus the
remaining content.  Supported formats: ``hermes`` (``<tool_call>{json}</tool_call>``),
``xml_fc`` (``<function_call><name>..</name><arguments>{json}</arguments></function_call>``),
``qwen3_coder`` (``<tool_call><function=name><parameter=k>v</parameter></function></tool_call>``),
``gpt_oss`` (``to=functions.name ... <|message|>{json}<|call|>``) and ``gemma4``
(fenced ``tool_code`` blocks with ``name(k=v, ...)`` calls).
"""

from __future__ import annotations

import ast
import json
import re
from dataclasses import dataclass, field


@dataclass
class ToolCall:
    name: str
    arguments: dict = field(default_factory=dict)


def _loads(s: str) -> dict:
    try:
        v = json.loads(s)
        return v if isinstance(v, dict) else {"value": v}
    except json.JSONDecodeError:
        return {"raw": s}


def parse_hermes(text: str):
    calls = []
    for m in re.finditer(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", text, re.S):
        d = _loads(m.group(1))
        calls.append(ToolCall(d.get("name", ""), d.get("arguments", {}) if isinstance(d.get("arguments"), dict)
                              else _loads(d.get("arguments", "{}"))))
    return calls, re.sub(r"<tool_call>.*?</tool_call>", "", text, flags=re.S).strip()


def parse_xml_fc(text: str):
    calls = []
    pat = r"<function_call>\s*<name>(.*?)</name>\s*<arguments>(.*?)</arguments>\s*</function_call>"
    for m in re.finditer(pat, text, re.S):
        calls.append(ToolCall(m.group(1).strip(), _loads(m.group(2).strip())))
    return calls, re.sub(r"<function_call>.*?</function_call>", "", text, flags=re.S).strip()


def parse_qwen3_coder(text: str):
    calls = []
    for m in re.finditer(r"<tool_call>\s*<function=([^>]+)>(.*?)</function>\s*</tool_call>", text, re.S):
        args = {}
        for p in re.finditer(r"<parameter=([^>]+)>(.*?)</parameter>", m.group(2), re.S):
            v = p.group(2).strip()
            try:
                args[p.group(1).strip()] = json.loads(v)
            except json.JSONDecodeError:
                args[p.group(1).strip()] = v
        calls.append(ToolCall(m.group(1).strip(), args))
    return calls, re.sub(r"<tool_call>.*?</tool_call>", "", text, flags=re.S).strip()


def parse_gpt_oss(text: str):
    calls = []
    for m in re.finditer(r"to=functions\.([\w\-.]+).*?<\|message\|>(.*?)<\|call\|>", text, re.S):
        calls.append(ToolCall(m.group(1), _loads(m.group(2).strip())))
    content = re.sub(r"<\|start\|>.*?<\|call\|>", "", text, flags=re.S)
    return calls, content.strip()


def parse_gemma4(text: str):
    calls = []
    for block in re.finditer(r"```tool_code\s*(.*?)```", text, re.S):
        for line in block.group(1).strip().splitlines():
            try:
                node = ast.parse(line.strip(), mode="eval").body
            except SyntaxError:
                continue
            if isinstance(node, ast.Call) and isinstance(node.func, ast.Name):
                args = {kw.arg: ast.literal_eval(kw.value) for kw in node.keywords}
                calls.append(ToolCall(node.func.id, args))
    return calls, re.sub(r"```tool_code.*?```", "", text, flags=re.S).strip()


PARSERS = {"hermes": parse_hermes, "xml_fc": parse_xml_fc, "qwen3_coder": parse_qwen3_coder,
           "gpt_oss": parse_gpt_oss, "gemma4": parse_gemma4}


def get_parser(name: str):
    if name not in PARSERS:
        raise KeyError(f"unknown tool parser {name!r}; have {sorted(PARSERS)}")
    return PARSERS[name]
