"""Per-step throughput and model-FLOPs-utilisation metrics, named as the
reference logs them (``perf/throughput`` in trained tokens per second per
GPU, ``perf/mfu/actor``, ``perf/time_per_step``, ``perf/total_num_tokens``;
``psrl/trainer/ppo/ray_trainer.py``).

MFU counts the actor update only: forward and backward matmul FLOPs (3x the
forward count of :func:`models.qwen.flops_per_token` at the step's mean
sequence length) over the training time and the trainer GPUs' peak
(``trainer.peak_tflops``, default the B200's 2250 dense bf16 TFLOP/s).
"""

from __future__ import annotations


def perf_metrics(cfg, args, tokens: int, num_trajectories: int, step_s: float, train_s: float, n_gpus: int,
                 n_train_gpus: int) -> dict:
    from ..models.qwen import flops_per_token
    out = {"perf/total_num_tokens": int(tokens), "perf/time_per_step": float(step_s)}
    if step_s > 0 and n_gpus > 0:
        out["perf/throughput"] = tokens / step_s / n_gpus
    if train_s > 0 and n_train_gpus > 0 and tokens > 0:
        mean_len = tokens / max(1, num_trajectories)
        flops = 3.0 * flops_per_token(args, int(mean_len)) * tokens
        peak = float(cfg.trainer.get("peak_tflops", 2250.0)) * 1e12
        out["perf/mfu/actor"] = flops / (train_s * n_train_gpus * peak)
    return out
