"""Configuration of the RL training-throughput benchmark (``bench.py``).

The workload is DAPO on a Qwen2.5-3B-shaped decoder at staleness 3 with 8
responses per prompt (preset ``dapo_qwen2.5_3b``).  Weak scaling: every GPU
adds ``prompts_per_gpu`` prompts to a step, so 8 GPUs run 128 prompts x 8
responses per step.
"""

from __future__ import annotations


def build_cfg(args, n_gpus: int):
    """Config for ``n_gpus`` GPUs from the parsed bench arguments
    (``prompts_per_gpu``, ``max_num_seqs``, ``kv_cache_gb``, ``recompute``,
    ``preset`` and ``override`` list)."""
    from ..config import load_config
    per_gpu = args.prompts_per_gpu
    ov = [
        f"psrl.staleness_buffer_entries={per_gpu * n_gpus}",
        "trainer.device=cuda",
        f"rollout.max_num_seqs={args.max_num_seqs}",
        f"++rollout.kv_cache_gb={args.kv_cache_gb}",
        "rollout.block_size=64",
        f"model.enable_gradient_checkpointing={'true' if args.recompute else 'false'}",
    ] + list(args.override)
    return load_config(preset=args.preset, overrides=ov)
