"""HF ↔ fused-layout parameter conversion and safetensors I/O (C18 converters).

HF Qwen2/Qwen3(-MoE) checkpoints store separate ``q_proj``/``k_proj``/``v_proj``
and ``gate_proj``/``up_proj`` (and per-expert matrices); this framework stacks
them (``attn.qkv``, ``mlp.gate_up``, ``experts_w13``/``experts_w2``).  The
conversion is a row split/concat along dim 0; the HF key names are the public
checkpoint format and must match exactly.
"""

from __future__ import annotations

import json
import os
import re

import torch

from .config import ModelArgs

_LAYER = re.compile(r"^layers\.(\d+)\.(.+)$")


def to_hf_state_dict(state: dict[str, torch.Tensor], a: ModelArgs) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    for k, t in state.items():
        m = _LAYER.match(k)
        if k == "embed.weight":
            out["model.embed_tokens.weight"] = t
        elif k == "norm":
            out["model.norm.weight"] = t
        elif k == "lm_head.weight":
            out["lm_head.weight"] = t
        elif k.startswith("value."):
            out["score." + k.split(".", 1)[1]] = t
        elif m:
            i, rest = m.group(1), m.group(2)
            p = f"model.layers.{i}."
            if rest == "ln1":
                out[p + "input_layernorm.weight"] = t
            elif rest == "ln2":
                out[p + "post_attention_layernorm.weight"] = t
            elif rest in ("attn.qkv.weight", "attn.qkv.bias"):
                kind = rest.rsplit(".", 1)[1]
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
                g, u = t.chunk(2, dim=0)
                out[p + "mlp.gate_proj.weight"] = g
                out[p + "mlp.up_proj.weight"] = u
            elif rest == "mlp.down.weight":
                out[p + "mlp.down_proj.weight"] = t
            elif rest == "mlp.router.weight":
                out[p + "mlp.gate.weight"] = t
            elif rest == "mlp.experts_w13":
                for e in range(t.shape[0]):
                    g, u = t[e].chunk(2, dim=0)
                    out[p + f"mlp.experts.{e}.gate_proj.weight"] = g
                    out[p + f"mlp.experts.{e}.up_proj.weight"] = u
            elif rest == "mlp.experts_w2":
                for e in range(t.shape[0]):
                    out[p + f"mlp.experts.{e}.down_proj.weight"] = t[e]
            else:
                raise KeyError(f"no HF mapping for {k}")
        else:
            raise KeyError(f"no HF mapping for {k}")
    return out


def from_hf_state_dict(hf: dict[str, torch.Tensor], a: ModelArgs) -> dict[str, torch.Tensor]:
    out: dict[str, torch.Tensor] = {}
    if "model.embed_tokens.weight" in hf:
        out["embed.weight"] = hf["model.embed_tokens.weight"]
    if "model.norm.weight" in hf:
        out["norm"] = hf["model.norm.weight"]
    if "lm_head.weight" in hf and not a.tie_word_embeddings:
        out["lm_head.weight"] = hf["lm_head.weight"]
    for k in ("score.weight", "score.bias"):
        if k in hf:
            out["value." + k.split(".", 1)[1]] = hf[k]
    for i in range(a.num_layers):
        p = f"model.layers.{i}."
        q = f"layers.{i}."
        out[q + "ln1"] = hf[p + "input_layernorm.weight"]
        out[q + "ln2"] = hf[p + "post_attention_layernorm.weight"]
        out[q + "attn.qkv.weight"] = torch.cat([hf[p + "self_attn.q_proj.weight"], hf[p + "self_attn.k_proj.weight"],
                                                hf[p + "self_attn.v_proj.weight"]], 0)
        if (p + "self_attn.q_proj.bias") in hf:
            out[q + "attn.qkv.bias"] = torch.cat([hf[p + "self_attn.q_proj.bias"], hf[p + "self_attn.k_proj.bias"],
                                                  hf[p + "self_attn.v_proj.bias"]], 0)
        out[q + "attn.o.weight"] = hf[p + "self_attn.o_proj.weight"]
        if a.qk_norm:
            out[q + "attn.q_norm"] = hf[p + "self_attn.q_norm.weight"]
            out[q + "attn.k_norm"] = hf[p + "self_attn.k_norm.weight"]
        if a.is_moe:
            out[q + "mlp.router.weight"] = hf[p + "mlp.gate.weight"]
            out[q + "mlp.experts_w13"] = torch.stack([
                torch.cat([hf[p + f"mlp.experts.{e}.gate_proj.weight"], hf[p + f"mlp.experts.{e}.up_proj.weight"]], 0)
                for e in range(a.num_experts)])
            out[q + "mlp.experts_w2"] = torch.stack([hf[p + f"mlp.experts.{e}.down_proj.weight"]
                                                     for e in range(a.num_experts)])
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
