"""Hot ops with sm_100a CUDA implementations and PyTorch references."""

from ._ext import ext, has_ext
from .activation import swiglu, swiglu_ref
from .debug import check_kernel_bounds, kernel_checks_enabled
from .attention import (
    paged_decode_attention,
    paged_prefill_attention,
    varlen_attention,
    varlen_attention_ref,
)
from .logprob import linear_logprob, linear_logprob_ref, logits_logprob
from .norm import head_rms_norm, rms_norm, rms_norm_ref
from .optim import NormAccumulator, adamw_, adamw_ref
from .rope import rope_qkv, rope_qkv_, rope_tables
from .sampling import sample, sample_ref

__all__ = [
    "NormAccumulator", "adamw_", "adamw_ref", "check_kernel_bounds", "ext", "has_ext", "head_rms_norm", "kernel_checks_enabled", "linear_logprob",
    "linear_logprob_ref", "logits_logprob", "paged_decode_attention", "paged_prefill_attention", "rms_norm",
    "rms_norm_ref", "rope_qkv", "rope_qkv_", "rope_tables", "sample", "sample_ref", "swiglu", "swiglu_ref",
    "varlen_attention", "varlen_attention_ref",
]
