"""Role placement on one node (C1/C4 resource pools).

Given the world size and ``psrl.deployment``, assigns every rank a role:
trainer ranks (one sharded-DP group, optionally TP-partitioned for the
Megatron-style backend), and rollout instances (each a group of
``rollout_ngpus_per_instance`` ranks, or heterogeneous per-instance TP sizes).
With one rank everything is colocated.  Reference:
``TaskRunner.init_resource_pool_mgr`` (``psrl/trainer/main_ppo.py:225-355``) and
``ResourcePoolManager`` (``psrl/trainer/ppo/utils.py:54``).
"""

from __future__ import annotations

import enum
from dataclasses import dataclass, field


class Role(enum.Enum):
    Actor = "actor"
    Critic = "critic"
    RefPolicy = "ref"
    Rollout = "rollout"
    Validate = "validate"


@dataclass
class RolloutInstanceSpec:
    instance_id: tuple
    ranks: list
    tp: int


@dataclass
class Placement:
    world: int
    train_ranks: list
    instances: list = field(default_factory=list)
    colocated: bool = False

    def role_of(self, rank: int) -> Role:
        if rank in self.train_ranks:
            return Role.Actor
        return Role.Rollout

    def instance_of(self, rank: int) -> RolloutInstanceSpec | None:
        for inst in self.instances:
            if rank in inst.ranks:
                return inst
        return None


def plan_placement(world: int, deployment) -> Placement:
    get = deployment.get if hasattr(deployment, "get") else (lambda k, d=None: d)
    if world == 1:
        return Placement(1, [0], [RolloutInstanceSpec((0, 0), [0], 1)], colocated=True)
    n_train = int(get("train_ngpus", 0) or 0)
    if n_train <= 0 or n_train >= world:
        n_train = max(1, world // 2)
    rest = list(range(n_train, world))
    het = get("heterogeneous_rollout", None)
    tps: list[int]
    if het is not None and het.get("enable"):
        tps = [int(x) for x in het.get("tensor_model_parallel_size_per_instance", [])]
        if sum(tps) != len(rest):
            raise ValueError(f"heterogeneous TP sizes {tps} do not cover {len(rest)} rollout GPUs")
    else:
        tp = int(get("rollout_ngpus_per_instance", 1) or 1)
        if len(rest) % tp:
            raise ValueError(f"{len(rest)} rollout GPUs not divisible by instance size {tp}")
        tps = [tp] * (len(rest) // tp)
    insts, k = [], 0
    for i, tp in enumerate(tps):
        insts.append(RolloutInstanceSpec((i, 0), rest[k:k + tp], tp))
        k += tp
    return Placement(world, list(range(n_train)), insts)
