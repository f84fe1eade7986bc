"""HF ↔ fused-layout parameter conversion and safetensors I/O (C18 converters).

HF checkpoints store separate ``q_proj``/``k_proj``/``v_proj`` and
``gate_proj``/``up_proj`` (Phi-3 stores them fused) and per-expert matrices
(under ``block_sparse_moe`` with ``w1``/``w3``/``w2`` for Mixtral); this
framework stacks them (``attn.qkv``, ``mlp.gate_up``, ``experts_w13`` /
``experts_w2``).  The conversion is a row split/concat along dim 0 plus the
family's names (``models/families.py``); the HF key names are the public
checkpoint format and must match exactly.  Gemma checkpoints store RMSNorm
weights as ``w - 1`` (the norm multiplies by ``1 + w``); they are shifted on
the way in and out.
"""

from __future__ import annotations

import json
import os
import re

import torch

from .config import ModelArgs
from .families import family_of

_LAYER = re.compile(r"^layers\.(\d+)\.(.+)$")
_NORMS = ("ln1", "ln2", "attn.q_norm", "attn.k_norm")


def to_hf_state_dict(state: dict[str, torch.Tensor], a: ModelArgs) -> dict[str, torch.Tensor]:
    f = family_of(a)
    g_name, u_name, d_name = f.expert_names
    mp = f.moe_prefix
    out: dict[str, torch.Tensor] = {}
    for k, t in state.items():
        m = _LAYER.match(k)
        if k == "embed.weight":
            out["model.embed_tokens.weight"] = t
        elif k == "norm":
            out["model.norm.weight"] = t - f.norm_offset if f.norm_offset else t
        elif k == "lm_head.weight":
            out["lm_head.weight"] = t
        elif k.startswith("value."):
            out["score." + k.split(".", 1)[1]] = t
        elif m:
            i, rest = m.group(1), m.group(2)
            p = f"model.layers.{i}."
            if rest in _NORMS and f.norm_offset:
                t = t - f.norm_offset
            if rest == "ln1":
                out[p + "input_layernorm.weight"] = t
            elif rest == "ln2":
                out[p + "post_attention_layernorm.weight"] = t
            elif rest in ("attn.qkv.weight", "attn.qkv.bias"):
                kind = rest.rsplit(".", 1)[1]
                if f.fused_qkv:
                    out[p + f"self_attn.qkv_proj.{kind}"] = t
                else:
                    q, kk, v = t.split([a.q_size, a.kv_size, a.kv_size], dim=0)
                    out[p + f"self_attn.q_proj.{kind}"] = q
                    out[p + f"self_attn.k_proj.{kind}"] = kk
                    out[p + f"self_attn.v_proj.{kind}"] = v
            elif rest == "attn.o.weight":
                out[p + "self_attn.o_proj.weight"] = t
            elif rest == "attn.q_norm":
                out[p + "self_attn.q_norm.weight"] = t
            elif rest == "attn.k_norm":
                out[p + "self_attn.k_norm.weight"] = t
            elif rest == "mlp.gate_up.weight":
                if f.fused_gate_up:
                    out[p + "mlp.gate_up_proj.weight"] = t
                else:
                    g, u = t.chunk(2, dim=0)
                    out[p + "mlp.gate_proj.weight"] = g
                    out[p + "mlp.up_proj.weight"] = u
            elif rest == "mlp.down.weight":
                out[p + "mlp.down_proj.weight"] = t
            elif rest == "mlp.router.weight":
                out[p + f"{mp}.gate.weight"] = t
            elif rest == "mlp.experts_w13":
                for e in range(t.shape[0]):
                    g, u = t[e].chunk(2, dim=0)
                    out[p + f"{mp}.experts.{e}.{g_name}.weight"] = g
                    out[p + f"{mp}.experts.{e}.{u_name}.weight"] = u
            elif rest == "mlp.experts_w2":
                for e in range(t.shape[0]):
                    out[p + f"{mp}.experts.{e}.{d_name}.weight"] = t[e]
            elif rest == "mlp.shared_gate_up.weight":
                g, u = t.chunk(2, dim=0)
                out[p + "mlp.shared_expert.gate_proj.weight"] = g
                out[p + "mlp.shared_expert.up_proj.weight"] = u
            elif rest == "mlp.shared_down.weight":
                out[p + "mlp.shared_expert.down_proj.weight"] = t
            elif rest == "mlp.shared_gate.weight":
                out[p + "mlp.shared_expert_gate.weight"] = t
            else:
                raise KeyError(f"no HF mapping for {k}")
        else:
            raise KeyError(f"no HF mapping for {k}")
    return out


def from_hf_state_dict(hf: dict[str, torch.Tensor], a: ModelArgs) -> dict[str, torch.Tensor]:
    f = family_of(a)
    g_name, u_name, d_name = f.expert_names
    mp = f.moe_prefix

    def norm(t):
        return t + f.norm_offset if f.norm_offset else t

    out: dict[str, torch.Tensor] = {}
    if "model.embed_tokens.weight" in hf:
        out["embed.weight"] = hf["model.embed_tokens.weight"]
    if "model.norm.weight" in hf:
        out["norm"] = norm(hf["model.norm.weight"])
    if "lm_head.weight" in hf and not a.tie_word_embeddings:
        out["lm_head.weight"] = hf["lm_head.weight"]
    for k in ("score.weight", "score.bias"):
        if k in hf:
            out["value." + k.split(".", 1)[1]] = hf[k]
    for i in range(a.num_layers):
        p = f"model.layers.{i}."
        q = f"layers.{i}."
        out[q + "ln1"] = norm(hf[p + "input_layernorm.weight"])
        out[q + "ln2"] = norm(hf[p + "post_attention_layernorm.weight"])
        for kind in ("weight", "bias"):
            if f.fused_qkv:
                if (p + f"self_attn.qkv_proj.{kind}") in hf:
                    out[q + f"attn.qkv.{kind}"] = hf[p + f"self_attn.qkv_proj.{kind}"]
            elif (p + f"self_attn.q_proj.{kind}") in hf:
                out[q + f"attn.qkv.{kind}"] = torch.cat([hf[p + f"self_attn.{n}_proj.{kind}"] for n in "qkv"], 0)
        out[q + "attn.o.weight"] = hf[p + "self_attn.o_proj.weight"]
        if a.qk_norm or a.qk_norm_full:
            out[q + "attn.q_norm"] = norm(hf[p + "self_attn.q_norm.weight"])
            out[q + "attn.k_norm"] = norm(hf[p + "self_attn.k_norm.weight"])
        if a.is_moe:
            out[q + "mlp.router.weight"] = hf[p + f"{mp}.gate.weight"]
            out[q + "mlp.experts_w13"] = torch.stack([
                torch.cat([hf[p + f"{mp}.experts.{e}.{g_name}.weight"], hf[p + f"{mp}.experts.{e}.{u_name}.weight"]], 0)
                for e in range(a.num_experts)])
            out[q + "mlp.experts_w2"] = torch.stack([hf[p + f"{mp}.experts.{e}.{d_name}.weight"]
                                                     for e in range(a.num_experts)])
            if a.shared_expert_intermediate_size:
                out[q + "mlp.shared_gate_up.weight"] = torch.cat([hf[p + "mlp.shared_expert.gate_proj.weight"],
                                                                  hf[p + "mlp.shared_expert.up_proj.weight"]], 0)
                out[q + "mlp.shared_down.weight"] = hf[p + "mlp.shared_expert.down_proj.weight"]
                out[q + "mlp.shared_gate.weight"] = hf[p + "mlp.shared_expert_gate.weight"]
        elif f.fused_gate_up:
            out[q + "mlp.gate_up.weight"] = hf[p + "mlp.gate_up_proj.weight"]
            out[q + "mlp.down.weight"] = hf[p + "mlp.down_proj.weight"]
        else:
            out[q + "mlp.gate_up.weight"] = torch.cat([hf[p + "mlp.gate_proj.weight"], hf[p + "mlp.up_proj.weight"]], 0)
            out[q + "mlp.down.weight"] = hf[p + "mlp.down_proj.weight"]
    return out


def save_hf(model, path: str, max_shard_bytes: int = 5 << 30) -> list[str]:
    """Write ``config.json`` + safetensors shards (+ index) in HF format."""
    from safetensors.torch import save_file

    if getattr(model, "tp", None) is not None or \
            any(getattr(getattr(layer, "mlp", None), "ep", None) is not None for layer in model.layers):
        raise ValueError("save_hf needs the unsharded model: save a TP / EP worker through "
                         "utils.checkpoint.save_worker, which assembles the shards")
    os.makedirs(path, exist_ok=True)
    a: ModelArgs = model.args
    state = {k: v.detach().to("cpu").contiguous() for k, v in model.state_dict().items()}
    hf = to_hf_state_dict(state, a)
    with open(os.path.join(path, "config.json"), "w") as fh:
        json.dump(a.to_hf_config(), fh, indent=2)
    shards: list[dict] = [{}]
    size = 0
    for k, t in hf.items():
        nb = t.numel() * t.element_size()
        if size + nb > max_shard_bytes and shards[-1]:
            shards.append({})
            size = 0
        shards[-1][k] = t.contiguous()
        size += nb
    names = []
    if len(shards) == 1:
        names.append("model.safetensors")
        save_file(shards[0], os.path.join(path, names[0]), metadata={"format": "pt"})
    else:
        weight_map = {}
        for i, sh in enumerate(shards):
            nm = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
            save_file(sh, os.path.join(path, nm), metadata={"format": "pt"})
            names.append(nm)
            for k in sh:
                weight_map[k] = nm
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as fh:
            json.dump({"metadata": {}, "weight_map": weight_map}, fh)
    return names


def load_hf_into(model, path: str) -> None:
    from safetensors.torch import load_file

    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    hf = {}
    for f in files:
        hf.update(load_file(os.path.join(path, f)))
    fused = from_hf_state_dict(hf, model.args)
    own = dict(model.named_parameters())
    with torch.no_grad():
        for k, t in fused.items():
            if k in own:
                own[k].copy_(t.to(own[k].dtype))
