"""Hierarchical configuration tree with attribute access, dotted overrides and
``${a.b}`` interpolation.

The reference composes its configuration with Hydra/OmegaConf
(``psrl/trainer/config/ppo_trainer.yaml:2-48``, ``psrl/trainer/config/psrl/psrl.yaml:1-24``)
and is driven from the command line with ``key=value`` / ``++key=value`` overrides.
Neither Hydra nor OmegaConf is part of this framework's dependency set, so this
module provides the small subset that the framework relies on:

* nested mapping with attribute access (``cfg.psrl.staleness``),
* deep merge of YAML files (group composition),
* ``a.b.c=value`` / ``+a.b=value`` / ``++a.b=value`` overrides parsed with YAML scalars,
* ``${a.b}`` interpolation resolved lazily against the root.
"""

from __future__ import annotations

import copy
import re
from collections.abc import Iterable, Mapping
from pathlib import Path
from typing import Any

import yaml

_INTERP = re.compile(r"\$\{([^}]+)\}")


class ConfigNode(dict):
    """A dict whose keys are also attributes; nested dicts become nodes."""

    def __init__(self, data: Mapping | None = None, _root: "ConfigNode | None" = None):
        super().__init__()
        object.__setattr__(self, "_root", _root)
        for k, v in (data or {}).items():
            self[k] = v

    # -- structure -------------------------------------------------------------
    def _wrap(self, value):
        root = self._root if self._root is not None else self
        if isinstance(value, ConfigNode):
            value = dict(value)
        if isinstance(value, Mapping):
            return ConfigNode(value, _root=root)
        if isinstance(value, list):
            return [self._wrap(v) for v in value]
        return value

    def __setitem__(self, key, value):
        super().__setitem__(key, self._wrap(value))

    def __getattr__(self, key):
        try:
            return self[key]
        except KeyError as exc:
            raise AttributeError(key) from exc

    def __setattr__(self, key, value):
        self[key] = value

    def __getitem__(self, key):
        value = super().__getitem__(key)
        return self._resolve(value)

    def get(self, key, default=None):
        if key in self:
            return self[key]
        return default

    def __deepcopy__(self, memo):
        return ConfigNode(copy.deepcopy(self.to_dict(resolve=False), memo))

    def __reduce__(self):
        # a root pickles its raw tree (interpolations stay live); a sub-node
        # pickles resolved values, since its root does not travel with it
        return ConfigNode, (self.to_dict(resolve=self._root is not None),)

    # -- interpolation ---------------------------------------------------------
    def _resolve(self, value, _depth: int = 0):
        if not isinstance(value, str) or "${" not in value:
            return value
        if _depth > 16:
            raise ValueError(f"interpolation too deep while resolving {value!r}")
        root = self._root if self._root is not None else self
        full = _INTERP.fullmatch(value)
        if full:
            return root._resolve(root.select(full.group(1)), _depth + 1)
        return _INTERP.sub(lambda m: str(root._resolve(root.select(m.group(1)), _depth + 1)), value)

    def select(self, dotted: str, default: Any = KeyError):
        node: Any = self
        for part in dotted.split("."):
            if isinstance(node, ConfigNode) and dict.__contains__(node, part):
                node = dict.__getitem__(node, part)
            else:
                if default is KeyError:
                    raise KeyError(dotted)
                return default
        return node

    # -- conversion ------------------------------------------------------------
    def to_dict(self, resolve: bool = True) -> dict:
        out = {}
        for k in self.keys():
            v = self[k] if resolve else dict.__getitem__(self, k)
            if isinstance(v, ConfigNode):
                v = v.to_dict(resolve)
            elif isinstance(v, list):
                v = [x.to_dict(resolve) if isinstance(x, ConfigNode) else x for x in v]
            out[k] = v
        return out

    def to_yaml(self) -> str:
        return yaml.safe_dump(self.to_dict(), sort_keys=False)


def deep_merge(base: dict, other: Mapping) -> dict:
    """Recursively merge ``other`` into ``base`` (in place) and return ``base``."""
    for k, v in other.items():
        if isinstance(v, Mapping) and isinstance(base.get(k), Mapping):
            base[k] = deep_merge(dict(base[k]), v)
        else:
            base[k] = copy.deepcopy(v)
    return base


def load_yaml(path: str | Path) -> dict:
    with open(path) as fh:
        return yaml.safe_load(fh) or {}


def parse_override(text: str) -> tuple[str, Any, bool]:
    """Parse ``[+|++]a.b.c=value`` into (path, value, may_create)."""
    create = False
    if text.startswith("++"):
        text, create = text[2:], True
    elif text.startswith("+"):
        text, create = text[1:], True
    if "=" not in text:
        raise ValueError(f"override {text!r} must look like key=value")
    key, raw = text.split("=", 1)
    value = yaml.safe_load(raw) if raw != "" else ""
    return key.strip(), value, create


def apply_overrides(cfg: ConfigNode, overrides: Iterable[str]) -> ConfigNode:
    for ov in overrides:
        key, value, create = parse_override(ov)
        parts = key.split(".")
        node = cfg
        for p in parts[:-1]:
            if p not in node:
                if not create:
                    raise KeyError(f"override {key!r}: unknown group {p!r} (use ++ to create)")
                node[p] = {}
            node = dict.__getitem__(node, p)
        if parts[-1] not in node and not create:
            raise KeyError(f"override {key!r}: unknown key (use ++ to create)")
        node[parts[-1]] = value
    return cfg
