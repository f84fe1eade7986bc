"""Model architecture arguments and presets.

One fused decoder covers every supported family; :class:`ModelArgs` holds the
switches (``models/families.py`` maps HF configs onto them)."""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field, fields, replace
from pathlib import Path


@dataclass
class ModelArgs:
    arch: str = "qwen2"                 # HF model_type of a registered family (models/families.py)
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_layers: int = 36
    num_heads: int = 16
    num_kv_heads: int = 2
    head_dim: int = 128
    intermediate_size: int = 11008
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    tie_word_embeddings: bool = True
    qkv_bias: bool = True               # Qwen2/2.5: True; Qwen3: False
    qk_norm: bool = False               # Qwen3: per-head RMSNorm on q and k
    max_position: int = 32768
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    router_zipf_alpha: float = 0.0      # >0: add log Zipf(alpha) prior to router logits (skewed load)
    value_head: bool = False            # critic: scalar head instead of the LM head
    # family switches
    rope_scaling: dict | None = None    # {"rope_type": "llama3" | "linear", "factor": ..., ...}
    qk_norm_full: bool = False          # OLMoE: RMSNorm over the whole q / k projection
    shared_expert_intermediate_size: int = 0   # Qwen2-MoE: always-on expert with a sigmoid gate
    hidden_act: str = "silu"            # silu (SwiGLU) | gelu_tanh (GeGLU, Gemma)
    embed_scale: float = 0.0            # Gemma: embeddings multiplied by sqrt(hidden)
    sliding_window: int | None = None   # Mistral: attention window (must cover the whole context)
    extra: dict = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def rope_spec(self):
        """Hashable RoPE description for the cos/sin table cache: the base, or
        (base, scaling items) when the family rescales frequencies."""
        if not self.rope_scaling:
            return float(self.rope_theta)
        return (float(self.rope_theta),) + tuple(sorted((k, v) for k, v in self.rope_scaling.items()
                                                        if not isinstance(v, (list, dict))))

    def check_context(self, length: int) -> None:
        """Sliding-window attention is implemented only as full attention, which
        is exact while the window covers the whole context."""
        if self.sliding_window is not None and length > self.sliding_window:
            raise NotImplementedError(f"context of {length} tokens exceeds the {self.sliding_window}-token "
                                      "sliding window; windowed attention is not implemented")

    def num_params(self) -> int:
        h, L = self.hidden_size, self.num_layers
        attn = h * self.qkv_size + (self.qkv_size if self.qkv_bias else 0) + self.q_size * h
        if self.is_moe:
            mlp = self.num_experts * 3 * h * self.moe_intermediate_size + self.num_experts * h
            mlp += 3 * h * self.shared_expert_intermediate_size + (h if self.shared_expert_intermediate_size else 0)
        else:
            mlp = 3 * h * self.intermediate_size
        norms = 2 * h + (2 * self.head_dim if self.qk_norm else 0) + (self.q_size + self.kv_size
                                                                       if self.qk_norm_full else 0)
        emb = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        return L * (attn + mlp + norms) + emb + h

    def active_params_per_token(self) -> int:
        """Matmul parameters touched per token (for FLOP accounting)."""
        h, L = self.hidden_size, self.num_layers
        attn = h * self.qkv_size + self.q_size * h
        if self.is_moe:
            mlp = self.num_experts_per_tok * 3 * h * self.moe_intermediate_size + self.num_experts * h
            mlp += 3 * h * self.shared_expert_intermediate_size
        else:
            mlp = 3 * h * self.intermediate_size
        return L * (attn + mlp) + self.vocab_size * h

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_hf_config(cls, cfg: dict) -> "ModelArgs":
        from .families import args_from_hf_config
        return args_from_hf_config(cfg)

    def to_hf_config(self) -> dict:
        from .families import hf_config_from_args
        return hf_config_from_args(self)


PRESETS: dict[str, ModelArgs] = {
    # 2-layer Qwen2-style decoder for CPU/gloo plumbing runs
    "tiny": ModelArgs(arch="qwen2", vocab_size=1024, hidden_size=256, num_layers=2, num_heads=4, num_kv_heads=2,
                      head_dim=64, intermediate_size=688, tie_word_embeddings=True, max_position=4096),
    # GPU test model: head_dim 128 so every CUDA kernel path is exercised
    "tiny128": ModelArgs(arch="qwen2", vocab_size=2048, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=2,
                         head_dim=128, intermediate_size=1024, tie_word_embeddings=True, max_position=8192),
    "qwen2.5-3b": ModelArgs(arch="qwen2", vocab_size=151936, hidden_size=2048, num_layers=36, num_heads=16,
                            num_kv_heads=2, head_dim=128, intermediate_size=11008, tie_word_embeddings=True),
    "qwen2.5-7b": ModelArgs(arch="qwen2", vocab_size=152064, hidden_size=3584, num_layers=28, num_heads=28,
                            num_kv_heads=4, head_dim=128, intermediate_size=18944, tie_word_embeddings=False),
    "qwen3-8b": ModelArgs(arch="qwen3", vocab_size=151936, hidden_size=4096, num_layers=36, num_heads=32,
                          num_kv_heads=8, head_dim=128, intermediate_size=12288, tie_word_embeddings=False,
                          qkv_bias=False, qk_norm=True),
    "qwen3-30b-a3b": ModelArgs(arch="qwen3_moe", vocab_size=151936, hidden_size=2048, num_layers=48, num_heads=32,
                               num_kv_heads=4, head_dim=128, intermediate_size=6144, tie_word_embeddings=False,
                               qkv_bias=False, qk_norm=True, num_experts=128, num_experts_per_tok=8,
                               moe_intermediate_size=768, router_zipf_alpha=1.1),
    "tiny-moe": ModelArgs(arch="qwen3_moe", vocab_size=2048, hidden_size=512, num_layers=2, num_heads=8,
                          num_kv_heads=2, head_dim=128, intermediate_size=1024, tie_word_embeddings=False,
                          qkv_bias=False, qk_norm=True, num_experts=8, num_experts_per_tok=2,
                          moe_intermediate_size=256, router_zipf_alpha=1.1, max_position=8192),
}


def model_args_from_config(model_cfg) -> ModelArgs:
    """Resolve ``model.preset`` / ``model.path`` (HF config.json) into ModelArgs."""
    path = model_cfg.get("path") if hasattr(model_cfg, "get") else None
    if path:
        with open(Path(path) / "config.json") as fh:
            return ModelArgs.from_hf_config(json.load(fh))
    preset = model_cfg.get("preset") or "tiny"
    if preset not in PRESETS:
        raise KeyError(f"unknown model preset {preset!r}; have {sorted(PRESETS)}")
    args = replace(PRESETS[preset])
    # ``model.overrides``: ModelArgs fields to change on the preset (a smaller
    # layer count for a test run, a longer max_position, ...)
    over = model_cfg.get("overrides", None) if hasattr(model_cfg, "get") else None
    if over:
        known = {f.name for f in fields(ModelArgs)}
        bad = sorted(set(over) - known)
        if bad:
            raise KeyError(f"model.overrides names unknown ModelArgs fields {bad}")
        args = replace(args, **{k: over[k] for k in over})
    return args
