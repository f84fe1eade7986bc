"""Megatron-style tensor parallelism for the trainer's dense decoder (K15,
baseline collectives).

With a tensor-parallel group of size P, rank r keeps

* attention: query heads [r nq/P, (r+1) nq/P) and KV heads [r nkv/P, ...) of
  the fused QKV projection (column parallel, bias sliced alike) and the
  matching input columns of the output projection (row parallel);
* MLP: intermediate columns [r I/P, (r+1) I/P) of both the gate and the up
  halves of ``gate_up`` (column parallel, still [gate | up] per rank) and the
  matching input columns of ``down`` (row parallel);
* MoE layers (expert tensor parallelism): the same column / row split of
  every expert's SwiGLU width and of the shared expert's; router and
  shared-expert gate replicated, their partial gradients summed over the
  group (:func:`make_tp_moe`);
* everything else (embedding, norms, q/k head norms, LM head) replicated.

A layer's input enters the column-parallel projections through
``copy_to_tp`` (identity forward, all-reduce of the gradient backward) and the
row-parallel outputs leave through ``reduce_from_tp`` (all-reduce forward,
identity backward), so replicated parameters see identical activations and
gradients on every rank.  The collectives are NCCL on GPU (the baseline path;
the GEMM-fused reduce-scatter / all-gather kernels are not built) and gloo on
CPU.  Shards are sliced from the full deterministically initialised model, so
TP and single-rank runs start from the same weights.

Reference: the Megatron TP layouts the reference converts
(``psrl/utils/megatron_converter.py``) and the 7B PPO recipe at TP=2.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops
from ..ops.linear import gate_up_swiglu, linear


@dataclass
class TPGroup:
    group: object
    world: int
    rank: int
    # fused GEMM + all-reduce over NVLink (parallel/tp_fused.py) for CUDA pairs;
    # None: local GEMM then an NCCL (or gloo) all-reduce
    fused: object = None

    def fused_fits(self, x, n_out: int) -> bool:
        f = self.fused
        return f is not None and x.is_cuda and x.reshape(-1, x.shape[-1]).shape[0] * n_out <= f.max_elems


def make_tp_group(group, device=None, fused_max_elems: int = 0) -> TPGroup:
    """TP group handle; with ``fused_max_elems`` > 0, a CUDA device and two
    ranks, the row-parallel GEMMs (and the column-parallel data gradients)
    run as fused GEMM + all-reduce kernels with accumulators of that size."""
    tp = TPGroup(group, dist.get_world_size(group), dist.get_rank(group))
    if fused_max_elems > 0 and tp.world == 2 and device is not None and torch.device(device).type == "cuda":
        from .tp_fused import FusedTP
        tp.fused = FusedTP(group, device, fused_max_elems)
    return tp


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        y = x.contiguous().clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x, tp: TPGroup):
    return _CopyToTP.apply(x, tp.group)


def reduce_from_tp(x, tp: TPGroup):
    return _ReduceFromTP.apply(x, tp.group)


class TPAttention(nn.Module):
    def __init__(self, full, tp: TPGroup):
        super().__init__()
        a = full.a
        if a.num_heads % tp.world or a.num_kv_heads % tp.world:
            raise ValueError(f"{a.num_heads} query / {a.num_kv_heads} KV heads do not split over TP={tp.world}")
        self.tp = tp
        self.a = a
        self.la = replace(a, num_heads=a.num_heads // tp.world, num_kv_heads=a.num_kv_heads // tp.world)
        d, r = a.head_dim, tp.rank
        qn, kn = self.la.num_heads * d, self.la.num_kv_heads * d
        rows = torch.cat([torch.arange(r * qn, (r + 1) * qn),
                          a.q_size + torch.arange(r * kn, (r + 1) * kn),
                          a.q_size + a.kv_size + torch.arange(r * kn, (r + 1) * kn)])
        w = full.qkv.weight.data
        self.qkv_weight = nn.Parameter(w.index_select(0, rows.to(w.device)).clone())
        self.qkv_bias = None
        if full.qkv.bias is not None:
            self.qkv_bias = nn.Parameter(full.qkv.bias.data.index_select(0, rows.to(w.device)).clone())
        self.o_weight = nn.Parameter(full.o.weight.data[:, r * qn:(r + 1) * qn].clone())
        if a.qk_norm:
            self.q_norm = nn.Parameter(full.q_norm.data.clone())
            self.k_norm = nn.Parameter(full.k_norm.data.clone())

    def forward(self, x, positions, cu_seqlens, max_seqlen):
        la = self.la
        T = x.shape[0]
        if self.tp.fused_fits(x, self.a.hidden_size):
            from .tp_fused import column_parallel
            qkv = column_parallel(x, self.qkv_weight, self.qkv_bias, self.tp.fused)
        else:
            x = copy_to_tp(x, self.tp)
            qkv = linear(x, self.qkv_weight, self.qkv_bias)
        if la.qk_norm:
            T = qkv.shape[0]
            q, k, v = qkv.split([la.q_size, la.kv_size, la.kv_size], dim=-1)
            q = ops.head_rms_norm(q.reshape(T, la.num_heads, la.head_dim), self.q_norm, la.rms_eps).reshape(T, -1)
            k = ops.head_rms_norm(k.reshape(T, la.num_kv_heads, la.head_dim), self.k_norm, la.rms_eps).reshape(T, -1)
            qkv = torch.cat([q, k, v], dim=-1)
        qkv = ops.rope_qkv(qkv.contiguous(), positions, la.num_heads, la.num_kv_heads, la.head_dim, la.rope_spec)
        o = ops.varlen_attention(qkv, cu_seqlens, max_seqlen, la.num_heads, la.num_kv_heads, la.head_dim)
        if self.tp.fused_fits(o, self.a.hidden_size) and T == o.shape[0]:
            from .tp_fused import row_parallel
            return row_parallel(o, self.o_weight, self.tp.fused)
        return reduce_from_tp(linear(o, self.o_weight), self.tp)


class TPMLP(nn.Module):
    def __init__(self, full, tp: TPGroup, intermediate: int):
        super().__init__()
        if intermediate % tp.world:
            raise ValueError(f"intermediate size {intermediate} does not split over TP={tp.world}")
        self.tp = tp
        il, r = intermediate // tp.world, tp.rank
        w = full.gate_up.weight.data
        self.gate_up_weight = nn.Parameter(torch.cat([w[r * il:(r + 1) * il], w[intermediate + r * il:
                                                                                   intermediate + (r + 1) * il]]).clone())
        self.down_weight = nn.Parameter(full.down.weight.data[:, r * il:(r + 1) * il].clone())

    def forward(self, x):
        hidden = self.down_weight.shape[0]
        if self.tp.fused_fits(x, hidden):
            from .tp_fused import column_parallel, row_parallel
            h = ops.swiglu(column_parallel(x, self.gate_up_weight, None, self.tp.fused))
            return row_parallel(h, self.down_weight, self.tp.fused)
        x = copy_to_tp(x, self.tp)
        return reduce_from_tp(linear(gate_up_swiglu(x, self.gate_up_weight), self.down_weight), self.tp)


def _sum_over_tp(tp: TPGroup):
    def hook(g):
        g = g.clone()
        dist.all_reduce(g, group=tp.group)
        return g
    return hook


def make_tp_moe(full, tp: TPGroup):
    """Expert tensor parallelism (ETP = TP): every expert's SwiGLU width, and
    the shared expert's, split over the TP ranks like a dense MLP (gate / up
    rows and the matching down columns of each expert); the router and the
    shared-expert gate are replicated.  Routing is identical on every rank, so
    each rank computes every routed (token, expert) pair at 1/P of the width
    and the partial outputs are summed by the layer's all-reduce.  The router
    and shared-gate gradients come out partial (each rank sees its own
    partial expert outputs) and are summed over the TP group by a gradient
    hook, which keeps them identical, as replicated parameters must be.
    Parameter names stay those of the unsharded MoE block."""
    from ..models.qwen import MoE
    a = full.a
    I, Is, P, r = a.moe_intermediate_size, a.shared_expert_intermediate_size, tp.world, tp.rank
    if I % P or Is % P:
        raise ValueError(f"expert width {I} / shared width {Is} does not split over TP={P}")

    class TPMoE(MoE):
        def forward(self, x):
            return reduce_from_tp(MoE.forward(self, copy_to_tp(x, self.tp)), self.tp)

    m = TPMoE.__new__(TPMoE)
    nn.Module.__init__(m)
    m.a, m.tp = a, tp
    il = I // P
    m.router = full.router
    w13, w2 = full.experts_w13.data, full.experts_w2.data
    m.experts_w13 = nn.Parameter(torch.cat([w13[:, r * il:(r + 1) * il], w13[:, I + r * il:I + (r + 1) * il]],
                                           dim=1).contiguous())
    m.experts_w2 = nn.Parameter(w2[:, :, r * il:(r + 1) * il].contiguous())
    m.register_buffer("router_prior", full.router_prior, persistent=False)
    m.router.weight.register_hook(_sum_over_tp(tp))
    names = ["experts_w13", "experts_w2"]
    if Is:
        sl = Is // P
        g = full.shared_gate_up.weight.data
        m.shared_gate_up = nn.Linear(a.hidden_size, 2 * sl, bias=False, device=g.device, dtype=g.dtype)
        m.shared_gate_up.weight.data.copy_(torch.cat([g[r * sl:(r + 1) * sl], g[Is + r * sl:Is + (r + 1) * sl]]))
        d = full.shared_down.weight.data
        m.shared_down = nn.Linear(sl, a.hidden_size, bias=False, device=d.device, dtype=d.dtype)
        m.shared_down.weight.data.copy_(d[:, r * sl:(r + 1) * sl])
        m.shared_gate = full.shared_gate
        m.shared_gate.weight.register_hook(_sum_over_tp(tp))
        names += ["shared_gate_up.weight", "shared_down.weight"]
    return m, names


@torch.no_grad()
def apply_tensor_parallel(model, tp: TPGroup) -> list[str]:
    """Shard every decoder layer of ``model`` in place (attention heads, the
    dense MLP's width, or each expert's width in a MoE layer); returns the
    names of the sharded parameters (the rest are replicated)."""
    a = model.args
    if a.qk_norm_full or a.hidden_act != "silu":
        raise NotImplementedError("tensor parallelism of full-width q/k norms or GeGLU is not implemented")
    names = []
    for i, layer in enumerate(model.layers):
        layer.attn = TPAttention(layer.attn, tp)
        names += [f"layers.{i}.attn.qkv_weight", f"layers.{i}.attn.o_weight"]
        if a.is_moe:
            layer.mlp, mnames = make_tp_moe(layer.mlp, tp)
            names += [f"layers.{i}.mlp.{n}" for n in mnames]
        else:
            layer.mlp = TPMLP(layer.mlp, tp, a.intermediate_size)
            names += [f"layers.{i}.mlp.gate_up_weight", f"layers.{i}.mlp.down_weight"]
        if layer.attn.qkv_bias is not None:
            names.append(f"layers.{i}.attn.qkv_bias")
    model.tp = tp
    return names


@torch.no_grad()
def engine_slices(name: str, shape: tuple, args, r: int, P: int) -> list[tuple[int, int, int]]:
    """(dim, start, length) pieces of the full tensor that make TP engine rank
    ``r``'s tensor, in :func:`shard_engine_tensors`'s layout: the trainer's TP
    layout (``models.converters.tp_slices``) for attention and the (shared)
    MLP, whole experts [r E/P, (r+1) E/P) for MoE, embeddings and everything
    else replicated."""
    from ..models.converters import tp_slices
    if name.endswith("experts_w13") or name.endswith("experts_w2"):
        per = shape[0] // P
        return [(0, r * per, per)]
    if name.endswith(("attn.qkv.weight", "attn.qkv.bias", "attn.o.weight", "mlp.gate_up.weight", "mlp.down.weight",
                      "mlp.shared_gate_up.weight", "mlp.shared_down.weight")):
        return tp_slices(name, shape, args, r, P)
    return [(0, 0, shape[0])]


def shard_engine_tensors(args, tensors: dict, tp: TPGroup) -> dict:
    """This TP rank's shard of full engine tensors (``layers.{i}.attn.qkv.weight``
    and so on), in the layout the TP trainer's shards and a TP rollout engine
    use; replicated tensors are shared, not copied."""
    d, r, P = args.head_dim, tp.rank, tp.world
    qn = args.num_heads // P * d
    if args.num_kv_heads >= P:
        kn, k0 = args.num_kv_heads // P * d, r * (args.num_kv_heads // P) * d
    else:
        # more ranks than KV heads: the KV head this rank's query heads read (replicated)
        kn, k0 = d, (r * args.num_kv_heads // P) * d
    il = args.intermediate_size // P
    rows = torch.cat([torch.arange(r * qn, (r + 1) * qn), args.q_size + torch.arange(k0, k0 + kn),
                      args.q_size + args.kv_size + torch.arange(k0, k0 + kn)])
    out = {}
    for n, t in tensors.items():
        if n.endswith("attn.qkv.weight") or n.endswith("attn.qkv.bias"):
            out[n] = t.index_select(0, rows.to(t.device)).contiguous()
        elif n.endswith("attn.o.weight"):
            out[n] = t[:, r * qn:(r + 1) * qn].contiguous()
        elif n.endswith("mlp.gate_up.weight"):
            I = args.intermediate_size
            out[n] = torch.cat([t[r * il:(r + 1) * il], t[I + r * il:I + (r + 1) * il]]).contiguous()
        elif n.endswith("mlp.down.weight"):
            out[n] = t[:, r * il:(r + 1) * il].contiguous()
        elif n.endswith("mlp.experts_w13") or n.endswith("mlp.experts_w2"):
            # expert parallelism over the TP group: whole experts [r E/P, (r+1) E/P)
            el = args.num_experts // P
            out[n] = t[r * el:(r + 1) * el].contiguous()
        elif n.endswith("mlp.shared_gate_up.weight"):
            Is = args.shared_expert_intermediate_size
            sl = Is // P
            out[n] = torch.cat([t[r * sl:(r + 1) * sl], t[Is + r * sl:Is + (r + 1) * sl]]).contiguous()
        elif n.endswith("mlp.shared_down.weight"):
            sl = args.shared_expert_intermediate_size // P
            out[n] = t[:, r * sl:(r + 1) * sl].contiguous()
        else:
            out[n] = t
    return out
