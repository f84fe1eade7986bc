"""Group- and buffer-stage post-processors (C27).

* ``no_filter`` keeps everything.
* ``dynamic_sampling_filter`` (DAPO) drops prompt groups whose metric has zero
  variance (all-correct or all-wrong groups carry no GRPO signal)
  (reference ``psrl/utils/post_processor/{group,buffer}_post_process/filter.py``).

A group processor sees one group's trajectories; a buffer processor sees a
whole READY buffer and returns the kept trajectories.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Callable

GROUP_PROCESSORS: dict[str, Callable] = {}
BUFFER_PROCESSORS: dict[str, Callable] = {}


def _metric(t, name: str):
    extra = t.meta.get("reward_extra", {}) if hasattr(t, "meta") else {}
    return extra.get(name, t.reward)


def group_processor(name):
    def deco(fn):
        GROUP_PROCESSORS[name] = fn
        return fn
    return deco


def buffer_processor(name):
    def deco(fn):
        BUFFER_PROCESSORS[name] = fn
        return fn
    return deco


@group_processor("no_filter")
def _g_keep(trajs, metric: str = "acc") -> bool:
    return True


@group_processor("dynamic_sampling_filter")
def _g_dynamic(trajs, metric: str = "acc") -> bool:
    vals = [_metric(t, metric) for t in trajs]
    return len(vals) < 2 or len(set(vals)) > 1


@buffer_processor("no_filter")
def _b_keep(trajs, metric: str = "acc"):
    return list(trajs)


@buffer_processor("dynamic_sampling_filter")
def _b_dynamic(trajs, metric: str = "acc"):
    groups = defaultdict(list)
    for t in trajs:
        groups[t.uid].append(t)
    out = []
    for g in groups.values():
        if _g_dynamic(g, metric):
            out.extend(g)
    return out
