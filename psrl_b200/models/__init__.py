"""Model definitions: Qwen2/2.5/3 dense and Qwen3-MoE decoders, critics."""

from .config import PRESETS, ModelArgs, model_args_from_config
from .qwen import QwenModel, build_model, flops_per_token, packed_positions

__all__ = ["ModelArgs", "PRESETS", "QwenModel", "build_model", "flops_per_token", "model_args_from_config",
           "packed_positions"]
