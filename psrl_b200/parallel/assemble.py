"""Full-model weights for a TP=1 rollout engine from a sharded trainer.

When the trainer shards parameters (expert parallelism: each rank owns E/P
experts of every layer; tensor parallelism: each rank owns head and
intermediate slices), a rollout engine beside it still needs every weight.
:class:`FullWeightAssembler` runs in two parts:

* ``gather()`` — a collective run on the trainer thread right after an optimizer step, under
  the process's exclusive weight lock.  It all-gathers every sharded parameter into a
  staging buffer of shape ``[P, *local_shape]``.
* ``assemble_into(engine_tensors)`` — local copies run on the rollout thread under the
  shared lock.  Replicated parameters are copied straight from the trainer.  Sharded ones
  are rearranged from the staging buffers into the engine's full tensors:
  - experts are concatenated along the expert dimension;
  - QKV rows are put back in q | k | v order;
  - gate_up rows are put back in gate | up order;
  - the O and down projections are concatenated along their input columns;
  - tensor-parallel experts (split along their width) get their gate, up and
    down slices put back per expert.

Engine tensor names are the unsharded model's (``layers.{i}.attn.qkv.weight``
and so on).  The gathers are NCCL on GPU and gloo on CPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

_TP_NAMES = {"attn.qkv_weight": "attn.qkv.weight", "attn.qkv_bias": "attn.qkv.bias",
             "attn.o_weight": "attn.o.weight", "mlp.gate_up_weight": "mlp.gate_up.weight",
             "mlp.down_weight": "mlp.down.weight"}


def engine_name(name: str) -> str:
    for k, v in _TP_NAMES.items():
        if name.endswith(k):
            return name[: -len(k)] + v
    return name


class FullWeightAssembler:
    def __init__(self, model, ep=None, tp=None, ep_names=(), tp_names=()):
        self.model = model
        self.args = model.args
        self.params = dict(model.named_parameters())
        self.ep, self.tp = ep, tp
        self.sharded: dict[str, tuple] = {}       # name -> (kind, group, world, staging)
        for n in ep_names:
            p = self.params[n]
            self.sharded[n] = ("ep", ep.group, ep.world, torch.empty((ep.world,) + tuple(p.shape), dtype=p.dtype,
                                                                     device=p.device))
        for n in tp_names:
            p = self.params[n]
            self.sharded[n] = ("tp", tp.group, tp.world, torch.empty((tp.world,) + tuple(p.shape), dtype=p.dtype,
                                                                     device=p.device))

    @torch.no_grad()
    def gather(self) -> None:
        for n, (_, group, world, st) in self.sharded.items():
            p = self.params[n].detach().contiguous()
            dist.all_gather_into_tensor(st.view(world * p.shape[0], *p.shape[1:]), p, group=group)

    @torch.no_grad()
    def assemble_into(self, engine: dict[str, torch.Tensor]) -> None:
        a = self.args
        for n, p in self.params.items():
            if n in self.sharded:
                continue
            t = engine.get(engine_name(n))
            if t is not None:
                t.copy_(p.detach(), non_blocking=True)
        for n, (kind, _, P, st) in self.sharded.items():
            dst = engine[engine_name(n)]
            if kind == "ep":
                dst.copy_(st.reshape(dst.shape), non_blocking=True)
                continue
            if n.endswith("attn.qkv_weight") or n.endswith("attn.qkv_bias"):
                qn = a.num_heads // P * a.head_dim
                kn = a.num_kv_heads // P * a.head_dim
                q, k, v = st.split([qn, kn, kn], dim=1)
                dst.copy_(torch.cat([q.reshape(P * qn, *q.shape[2:]), k.reshape(P * kn, *k.shape[2:]),
                                     v.reshape(P * kn, *v.shape[2:])]), non_blocking=True)
            elif n.endswith("mlp.gate_up_weight") or n.endswith("mlp.shared_gate_up.weight"):
                il = (a.intermediate_size if n.endswith("mlp.gate_up_weight") else a.shared_expert_intermediate_size) // P
                g, u = st.split([il, il], dim=1)
                dst.copy_(torch.cat([g.reshape(P * il, -1), u.reshape(P * il, -1)]), non_blocking=True)
            elif n.endswith("experts_w13"):
                # [P, E, 2 il, h] -> gate rows then up rows of every expert: [E, 2 P il, h]
                il = st.shape[2] // 2
                g, u = st.split([il, il], dim=2)
                E, h = st.shape[1], st.shape[3]
                dst.copy_(torch.cat([g.permute(1, 0, 2, 3).reshape(E, P * il, h),
                                     u.permute(1, 0, 2, 3).reshape(E, P * il, h)], dim=1), non_blocking=True)
            elif n.endswith("experts_w2"):
                # [P, E, h, il] -> [E, h, P il]
                dst.copy_(st.permute(1, 2, 0, 3).reshape(dst.shape), non_blocking=True)
            else:   # row-parallel O / down (and the shared expert's down): [P, h, cols] -> [h, P * cols]
                dst.copy_(st.permute(1, 0, 2).reshape(dst.shape), non_blocking=True)
