"""Model families: HF config ↔ :class:`ModelArgs` and HF checkpoint key names
(C18 converters; the reference's per-family parameter mappings and model
registry: ``psrl/utils/converter/modeling/vllm_modeling.py``,
``psrl/utils/converter/model_mappings.py:765``).

Every family runs on the same fused decoder (``models/qwen.py`` for training,
``rollout/engine.py`` for generation); a family is a set of architecture
switches on :class:`ModelArgs` plus the names its checkpoints use.  New
families register with :func:`register_family`.

Supported ``model_type`` values: ``qwen2``, ``qwen3``, ``qwen3_moe``,
``qwen2_moe`` (shared expert with a sigmoid gate), ``llama`` (incl. Llama-3
RoPE scaling), ``mistral`` (sliding window only where it spans the whole
context), ``mixtral``, ``olmoe`` (q/k RMSNorm over the full projection),
``phi3`` (fused ``qkv_proj`` / ``gate_up_proj`` in the checkpoint) and
``gemma`` (GeGLU, embeddings scaled by sqrt(hidden), RMSNorm weights stored as
``w - 1``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .config import ModelArgs


@dataclass(frozen=True)
class Family:
    model_type: str
    architecture: str                                 # HF ``architectures[0]``
    qkv_bias: bool = False
    qk_norm: str = ""                                 # "" | "head" | "full"
    fused_qkv: bool = False                           # checkpoint stores self_attn.qkv_proj
    fused_gate_up: bool = False                       # checkpoint stores mlp.gate_up_proj
    moe: bool = False
    moe_prefix: str = "mlp"                           # Mixtral: block_sparse_moe
    expert_names: tuple = ("gate_proj", "up_proj", "down_proj")
    shared_expert: bool = False
    norm_offset: float = 0.0                          # Gemma: checkpoint weight = ours - 1
    default_theta: float = 10000.0
    default_norm_topk: bool = True
    extra_hf: dict = field(default_factory=dict)      # fixed keys written to config.json


FAMILIES: dict[str, Family] = {}


def register_family(f: Family) -> Family:
    FAMILIES[f.model_type] = f
    return f


for _f in (
    Family("qwen2", "Qwen2ForCausalLM", qkv_bias=True, default_theta=1e6),
    Family("qwen3", "Qwen3ForCausalLM", qk_norm="head", default_theta=1e6),
    Family("qwen3_moe", "Qwen3MoeForCausalLM", qk_norm="head", moe=True, default_theta=1e6),
    Family("qwen2_moe", "Qwen2MoeForCausalLM", qkv_bias=True, moe=True, shared_expert=True,
           default_norm_topk=False, default_theta=1e6),
    Family("llama", "LlamaForCausalLM"),
    Family("mistral", "MistralForCausalLM"),
    Family("mixtral", "MixtralForCausalLM", moe=True, moe_prefix="block_sparse_moe",
           expert_names=("w1", "w3", "w2"), default_theta=1e6),
    Family("olmoe", "OlmoeForCausalLM", qk_norm="full", moe=True, default_norm_topk=False),
    Family("phi3", "Phi3ForCausalLM", fused_qkv=True, fused_gate_up=True),
    Family("gemma", "GemmaForCausalLM", norm_offset=1.0, extra_hf={"hidden_act": "gelu_pytorch_tanh"}),
):
    register_family(_f)


def family_of(a: ModelArgs) -> Family:
    try:
        return FAMILIES[a.arch]
    except KeyError:
        raise ValueError(f"unknown model family {a.arch!r}; registered: {sorted(FAMILIES)}") from None


def _rope(cfg: dict, default_theta: float) -> tuple[float, dict | None]:
    rp = cfg.get("rope_parameters") or {}
    theta = cfg.get("rope_theta", rp.get("rope_theta", default_theta))
    scaling = cfg.get("rope_scaling") or (rp if rp.get("rope_type", "default") != "default" else None)
    if scaling:
        kind = scaling.get("rope_type", scaling.get("type", "default"))
        if kind == "default":
            scaling = None
        elif kind not in ("llama3", "linear"):
            raise NotImplementedError(f"RoPE scaling {kind!r} is not implemented (llama3 and linear are)")
        else:
            scaling = {"rope_type": kind, **{k: v for k, v in scaling.items() if k not in ("rope_type", "type",
                                                                                          "rope_theta")}}
    if float(rp.get("partial_rotary_factor", cfg.get("partial_rotary_factor", 1.0))) != 1.0:
        raise NotImplementedError("partial rotary embeddings are not implemented")
    return float(theta), scaling


_TOKEN_KEYS = ("bos_token_id", "eos_token_id", "pad_token_id")


def args_from_hf_config(cfg: dict) -> ModelArgs:
    mt = cfg.get("model_type", "qwen2")
    if mt not in FAMILIES:
        raise ValueError(f"unsupported model_type {mt!r}; registered: {sorted(FAMILIES)}")
    f = FAMILIES[mt]
    heads = cfg["num_attention_heads"]
    theta, scaling = _rope(cfg, f.default_theta)
    act = cfg.get("hidden_activation") or cfg.get("hidden_act", "silu")
    act = {"silu": "silu", "swish": "silu", "gelu_pytorch_tanh": "gelu_tanh", "gelu": "gelu_tanh"}.get(act)
    if act is None:
        raise NotImplementedError(f"activation {cfg.get('hidden_act')!r} is not implemented")
    if cfg.get("mlp_bias"):
        raise NotImplementedError("MLP biases are not implemented")
    if cfg.get("clip_qkv"):
        raise NotImplementedError("clip_qkv is not implemented")
    if cfg.get("mlp_only_layers") or int(cfg.get("decoder_sparse_step", 1) or 1) != 1:
        raise NotImplementedError("interleaved dense / MoE layers are not implemented")
    window = cfg.get("sliding_window")
    if not cfg.get("use_sliding_window", mt in ("mistral",)) or not window:
        window = None
    n_exp = int(cfg.get("num_experts", cfg.get("num_local_experts", 0)) or 0) if f.moe else 0
    a = ModelArgs(
        arch=mt,
        vocab_size=cfg["vocab_size"],
        hidden_size=cfg["hidden_size"],
        num_layers=cfg["num_hidden_layers"],
        num_heads=heads,
        num_kv_heads=cfg.get("num_key_value_heads") or heads,
        head_dim=cfg.get("head_dim") or cfg["hidden_size"] // heads,
        intermediate_size=0 if f.moe and mt == "mixtral" else cfg.get("intermediate_size", 0),
        rope_theta=theta,
        rope_scaling=scaling,
        rms_eps=cfg.get("rms_norm_eps", 1e-6),
        tie_word_embeddings=bool(cfg.get("tie_word_embeddings", False)),
        qkv_bias=f.qkv_bias or bool(cfg.get("attention_bias", False)),
        qk_norm=f.qk_norm == "head",
        qk_norm_full=f.qk_norm == "full",
        max_position=cfg.get("max_position_embeddings", 32768),
        num_experts=n_exp,
        num_experts_per_tok=int(cfg.get("num_experts_per_tok", 0)) if f.moe else 0,
        moe_intermediate_size=(cfg.get("moe_intermediate_size") or cfg.get("intermediate_size", 0)) if f.moe else 0,
        norm_topk_prob=bool(cfg.get("norm_topk_prob", f.default_norm_topk)),
        shared_expert_intermediate_size=int(cfg.get("shared_expert_intermediate_size", 0)) if f.shared_expert else 0,
        hidden_act=act,
        embed_scale=float(cfg["hidden_size"]) ** 0.5 if mt == "gemma" else 0.0,
        sliding_window=window,
        extra={"hf_tokens": {k: cfg[k] for k in _TOKEN_KEYS if cfg.get(k) is not None}},
    )
    return a


def hf_config_from_args(a: ModelArgs) -> dict:
    f = family_of(a)
    d = {
        "model_type": f.model_type,
        "architectures": [f.architecture],
        "vocab_size": a.vocab_size,
        "hidden_size": a.hidden_size,
        "num_hidden_layers": a.num_layers,
        "num_attention_heads": a.num_heads,
        "num_key_value_heads": a.num_kv_heads,
        "head_dim": a.head_dim,
        "intermediate_size": a.moe_intermediate_size if f.model_type == "mixtral" else a.intermediate_size,
        "rope_theta": a.rope_theta,
        "rms_norm_eps": a.rms_eps,
        "tie_word_embeddings": a.tie_word_embeddings,
        "max_position_embeddings": a.max_position,
        "hidden_act": "gelu_pytorch_tanh" if a.hidden_act == "gelu_tanh" else "silu",
        "torch_dtype": "bfloat16",
    }
    if a.rope_scaling:
        d["rope_scaling"] = dict(a.rope_scaling)
    if f.model_type in ("llama", "mistral", "olmoe", "gemma", "qwen3", "qwen3_moe"):
        d["attention_bias"] = bool(a.qkv_bias)
    if f.model_type in ("mistral", "mixtral", "qwen2", "qwen2_moe", "phi3"):
        d["sliding_window"] = a.sliding_window
        if f.model_type in ("qwen2", "qwen2_moe"):
            d["use_sliding_window"] = a.sliding_window is not None
    if a.is_moe:
        key = "num_local_experts" if f.model_type == "mixtral" else "num_experts"
        d.update({key: a.num_experts, "num_experts_per_tok": a.num_experts_per_tok,
                  "norm_topk_prob": a.norm_topk_prob})
        if f.model_type != "mixtral":
            d["moe_intermediate_size"] = a.moe_intermediate_size
        if f.model_type == "olmoe":
            d["intermediate_size"] = a.moe_intermediate_size
    if f.shared_expert:
        d["shared_expert_intermediate_size"] = a.shared_expert_intermediate_size
        d["decoder_sparse_step"] = 1
        d["mlp_only_layers"] = []
    d.update(f.extra_hf)
    d.update((a.extra or {}).get("hf_tokens", {}))
    return d
