"""The fused decoder for training: Qwen2 / Qwen2.5 / Qwen3 / Qwen3-MoE /
Qwen2-MoE / Llama / Mistral / Mixtral / OLMoE / Phi-3 / Gemma (the family
switches are in :class:`ModelArgs`, the checkpoint names in
``models/families.py`` and ``models/hf_io.py``).

Parameter layout (shared with the rollout engine at TP=1):

* ``layers.{i}.attn.qkv.weight`` [(nq + 2 nkv) * d, h] — q, k, v rows stacked
  (HF ``q_proj``/``k_proj``/``v_proj``), optional ``qkv.bias``;
* ``layers.{i}.mlp.gate_up.weight`` [2 I, h] — HF ``gate_proj`` then ``up_proj``;
* MoE: ``layers.{i}.mlp.router.weight`` [E, h], ``experts_w13`` [E, 2 I_e, h],
  ``experts_w2`` [E, h, I_e].

Fusing at the parameter level makes every projection a single GEMM and lets
the trainer → rollout weight sync copy contiguous row ranges; HF checkpoints
are split/merged by :mod:`psrl_b200.models.hf_io`.

The forward runs over a packed (remove-padding) batch: ``input_ids`` [T],
``positions`` [T], ``cu_seqlens`` [B+1].  Hot ops go through
:mod:`psrl_b200.ops` (sm_100a kernels on GPU): the projections run on the
paired-CTA tcgen05 GEMM (:mod:`psrl_b200.ops.linear`, SwiGLU fused into the
gate_up epilogue), the ``nn.Linear`` modules only hold the parameters.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from .. import ops
from ..ops.linear import gate_up_swiglu, linear
from ..parallel.cp import CPPlan, cp_attention
from ..parallel.ulysses import UlyssesPlan, ulysses_attention
from .config import ModelArgs


class Attention(nn.Module):
    def __init__(self, a: ModelArgs):
        super().__init__()
        self.a = a
        self.qkv = nn.Linear(a.hidden_size, a.qkv_size, bias=a.qkv_bias)
        self.o = nn.Linear(a.q_size, a.hidden_size, bias=False)
        if a.qk_norm:
            self.q_norm = nn.Parameter(torch.ones(a.head_dim))
            self.k_norm = nn.Parameter(torch.ones(a.head_dim))
        elif a.qk_norm_full:
            self.q_norm = nn.Parameter(torch.ones(a.q_size))
            self.k_norm = nn.Parameter(torch.ones(a.kv_size))

    def forward(self, x, positions, cu_seqlens, max_seqlen):
        a = self.a
        qkv = linear(x, self.qkv.weight, self.qkv.bias)
        if a.qk_norm:
            T = qkv.shape[0]
            q, k, v = qkv.split([a.q_size, a.kv_size, a.kv_size], dim=-1)
            q = ops.head_rms_norm(q.reshape(T, a.num_heads, a.head_dim), self.q_norm, a.rms_eps).reshape(T, -1)
            k = ops.head_rms_norm(k.reshape(T, a.num_kv_heads, a.head_dim), self.k_norm, a.rms_eps).reshape(T, -1)
            qkv = torch.cat([q, k, v], dim=-1)
        elif a.qk_norm_full:
            q, k, v = qkv.split([a.q_size, a.kv_size, a.kv_size], dim=-1)
            q, _ = ops.rms_norm(q.contiguous(), self.q_norm, a.rms_eps)
            k, _ = ops.rms_norm(k.contiguous(), self.k_norm, a.rms_eps)
            qkv = torch.cat([q, k, v], dim=-1)
        qkv = ops.rope_qkv(qkv.contiguous(), positions, a.num_heads, a.num_kv_heads, a.head_dim, a.rope_spec)
        if isinstance(cu_seqlens, CPPlan):
            # context parallel: this rank's query chunks over the gathered keys
            o = cp_attention(qkv[:, : a.q_size], qkv[:, a.q_size:], cu_seqlens, a.num_heads, a.num_kv_heads,
                             a.head_dim)
        elif isinstance(cu_seqlens, UlyssesPlan):
            # Ulysses: all-to-all to head-parallel attention over the whole micro-batch and back
            o = ulysses_attention(qkv[:, : a.q_size], qkv[:, a.q_size:], cu_seqlens, a.num_heads,
                                  a.num_kv_heads, a.head_dim)
        else:
            o = ops.varlen_attention(qkv, cu_seqlens, max_seqlen, a.num_heads, a.num_kv_heads, a.head_dim)
        return linear(o, self.o.weight)


def gated_act(x: torch.Tensor, w_gate_up: torch.Tensor, act: str) -> torch.Tensor:
    """act(x W_gate^T) * (x W_up^T) for the fused [2I, h] gate_up weight:
    SwiGLU in the GEMM epilogue, GeGLU (tanh GELU, Gemma) after it."""
    if act == "silu":
        return gate_up_swiglu(x, w_gate_up)
    g, u = linear(x, w_gate_up).chunk(2, dim=-1)
    return F.gelu(g.float(), approximate="tanh").to(g.dtype) * u


class MLP(nn.Module):
    def __init__(self, a: ModelArgs):
        super().__init__()
        self.act = a.hidden_act
        self.gate_up = nn.Linear(a.hidden_size, 2 * a.intermediate_size, bias=False)
        self.down = nn.Linear(a.intermediate_size, a.hidden_size, bias=False)

    def forward(self, x):
        return linear(gated_act(x, self.gate_up.weight, self.act), self.down.weight)


def zipf_prior(num_experts: int, alpha: float, seed: int = 1234) -> torch.Tensor:
    """log of a Zipf(alpha) distribution over experts in a fixed random order."""
    ranks = torch.arange(1, num_experts + 1, dtype=torch.float64)
    p = ranks.pow(-alpha)
    p = p / p.sum()
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_experts, generator=g)
    return p.log()[perm].float()


class MoE(nn.Module):
    """Top-k routed SwiGLU experts (Qwen3-MoE: softmax router, renormalised top-k)."""

    def __init__(self, a: ModelArgs):
        super().__init__()
        self.a = a
        E, h, I = a.num_experts, a.hidden_size, a.moe_intermediate_size
        self.router = nn.Linear(h, E, bias=False)
        self.experts_w13 = nn.Parameter(torch.empty(E, 2 * I, h))
        self.experts_w2 = nn.Parameter(torch.empty(E, h, I))
        prior = zipf_prior(E, a.router_zipf_alpha) if a.router_zipf_alpha > 0 else torch.zeros(E)
        self.register_buffer("router_prior", prior, persistent=False)
        Is = a.shared_expert_intermediate_size
        if Is:
            # Qwen2-MoE: an always-on SwiGLU expert scaled by sigmoid(x w_gate)
            self.shared_gate_up = nn.Linear(h, 2 * Is, bias=False)
            self.shared_down = nn.Linear(Is, h, bias=False)
            self.shared_gate = nn.Linear(h, 1, bias=False)

    def shared(self, x):
        y = linear(gate_up_swiglu(x, self.shared_gate_up.weight), self.shared_down.weight)
        return torch.sigmoid(F.linear(x, self.shared_gate.weight).float()).to(y.dtype) * y

    def route(self, x):
        logits = self.router(x).float() + self.router_prior
        probs = logits.softmax(-1)
        w, idx = probs.topk(self.a.num_experts_per_tok, dim=-1)
        if self.a.norm_topk_prob:
            w = w / w.sum(-1, keepdim=True)
        return w, idx

    def forward(self, x):
        y = self.routed(x)
        return y + self.shared(x) if self.a.shared_expert_intermediate_size else y

    def routed(self, x):
        from ..ops import moe as moe_ops
        ep = getattr(self, "ep", None)
        if ep is not None:
            # expert parallel: this rank holds experts [ep.first, ep.first + ep.local)
            from ..parallel.ep import moe_forward_ep
            w, idx = self.route(x)
            return moe_forward_ep(x, w, idx, self.experts_w13, self.experts_w2, ep)
        if moe_ops.supported(x, self.experts_w13, self.experts_w2):
            return moe_ops.moe_mlp(x, self.router(x).float(), self.router_prior, self.experts_w13, self.experts_w2,
                                   self.a.num_experts_per_tok, bool(self.a.norm_topk_prob))
        from ..parallel.moe import moe_forward_local
        w, idx = self.route(x)
        return moe_forward_local(x, w.to(x.dtype), idx, self.experts_w13, self.experts_w2)


class DecoderLayer(nn.Module):
    def __init__(self, a: ModelArgs):
        super().__init__()
        self.a = a
        self.ln1 = nn.Parameter(torch.ones(a.hidden_size))
        self.ln2 = nn.Parameter(torch.ones(a.hidden_size))
        self.attn = Attention(a)
        self.mlp = MoE(a) if a.is_moe else MLP(a)

    def forward(self, x, resid, positions, cu_seqlens, max_seqlen):
        h, resid = ops.rms_norm(x, self.ln1, self.a.rms_eps, residual=resid)
        if resid is None:
            resid = x
        attn_out = self.attn(h, positions, cu_seqlens, max_seqlen)
        h2, resid = ops.rms_norm(attn_out, self.ln2, self.a.rms_eps, residual=resid)
        return self.mlp(h2), resid


class QwenModel(nn.Module):
    """Decoder trunk + (tied) LM head, or a scalar value head for critics."""

    def __init__(self, a: ModelArgs):
        super().__init__()
        self.args = a
        self.embed = nn.Embedding(a.vocab_size, a.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(a) for _ in range(a.num_layers)])
        self.norm = nn.Parameter(torch.ones(a.hidden_size))
        if a.value_head:
            self.value = nn.Linear(a.hidden_size, 1, bias=True)
        elif not a.tie_word_embeddings:
            self.lm_head = nn.Linear(a.hidden_size, a.vocab_size, bias=False)
        self.gradient_checkpointing = False

    # ------------------------------------------------------------------ init
    @torch.no_grad()
    def init_weights(self, seed: int = 0, std: float = 0.02) -> None:
        """Random init (normal(0, std) matrices, unit norms, zero biases),
        deterministic across processes for a given seed."""
        for i, (name, p) in enumerate(self.named_parameters()):
            if name.endswith(("ln1", "ln2", "norm", "q_norm", "k_norm")):
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                # one generator per tensor on the tensor's device: same values on every rank
                g = torch.Generator(device=p.device).manual_seed(seed * 100003 + i)
                t = torch.empty(p.shape, dtype=torch.float32, device=p.device).normal_(0.0, std, generator=g)
                p.copy_(t)

    def lm_head_weight(self) -> torch.Tensor:
        return self.embed.weight if self.args.tie_word_embeddings else self.lm_head.weight

    # --------------------------------------------------------------- forward
    def hidden_states(self, input_ids, positions, cu_seqlens, max_seqlen):
        a = self.args
        if a.sliding_window is not None and not isinstance(cu_seqlens, (CPPlan, UlyssesPlan)):
            a.check_context(int(max_seqlen))
        x = self.embed(input_ids)
        if a.embed_scale:
            x = x * torch.tensor(a.embed_scale, dtype=x.dtype)
        resid = None
        for layer in self.layers:
            if self.gradient_checkpointing and torch.is_grad_enabled():
                x, resid = checkpoint(layer, x, resid, positions, cu_seqlens, max_seqlen, use_reentrant=False)
            else:
                x, resid = layer(x, resid, positions, cu_seqlens, max_seqlen)
        h, _ = ops.rms_norm(x, self.norm, self.args.rms_eps, residual=resid)
        return h

    def logprobs(self, input_ids, positions, cu_seqlens, max_seqlen, labels, temperature: float = 1.0):
        """(log pi(label_t | prefix), entropy_t), fp32 [T]; labels < 0 are ignored."""
        h = self.hidden_states(input_ids, positions, cu_seqlens, max_seqlen)
        return ops.linear_logprob(h, self.lm_head_weight(), labels, temperature)

    def values(self, input_ids, positions, cu_seqlens, max_seqlen):
        h = self.hidden_states(input_ids, positions, cu_seqlens, max_seqlen)
        return self.value(h).float().squeeze(-1)

    def logits(self, input_ids, positions, cu_seqlens, max_seqlen):
        h = self.hidden_states(input_ids, positions, cu_seqlens, max_seqlen)
        return F.linear(h, self.lm_head_weight())


def build_model(a: ModelArgs, device="cpu", dtype=torch.float32, seed: int = 0) -> QwenModel:
    with torch.device("meta"):
        m = QwenModel(a)
    m = m.to_empty(device=device)
    m.init_weights(seed)
    m.to(dtype)
    if a.is_moe:
        for layer in m.layers:
            layer.mlp.router_prior = (zipf_prior(a.num_experts, a.router_zipf_alpha) if a.router_zipf_alpha > 0
                                      else torch.zeros(a.num_experts)).to(device)
    return m


def packed_positions(seqlens: list[int], device) -> tuple[torch.Tensor, torch.Tensor, int]:
    """positions [T] (int32) and cu_seqlens [B+1] (int32) for a packed batch."""
    cu = [0]
    for n in seqlens:
        cu.append(cu[-1] + n)
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in seqlens]) if seqlens else torch.zeros(0, dtype=torch.int32)
    return pos.to(device), torch.tensor(cu, dtype=torch.int32, device=device), max(seqlens) if seqlens else 0


def flops_per_token(a: ModelArgs, seq_len: int) -> float:
    """Forward matmul FLOPs per token (2 * params touched + causal attention)."""
    attn = 2 * 2 * a.num_layers * a.q_size * seq_len / 2 * 1.0
    return 2.0 * a.active_params_per_token() + attn


__all__ = ["Attention", "DecoderLayer", "MLP", "MoE", "QwenModel", "build_model", "flops_per_token",
           "packed_positions", "zipf_prior", "math"]
