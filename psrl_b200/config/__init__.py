"""Configuration loading, composition and validation.

Mirrors the reference's Hydra composition (``psrl/trainer/config/ppo_trainer.yaml``)
plus ``validate_config`` (``psrl/utils/config.py:94-389``) with a dependency-free
implementation (:mod:`psrl_b200.config.node`).
"""

from __future__ import annotations

from pathlib import Path
from typing import Iterable

from .node import ConfigNode, apply_overrides, deep_merge, load_yaml, parse_override

_HERE = Path(__file__).resolve().parent
DEFAULT_YAML = _HERE / "default.yaml"
PRESET_DIR = _HERE / "presets"


def load_config(
    path: str | Path | None = None, overrides: Iterable[str] = (), preset: str | None = None
) -> ConfigNode:
    """Compose default.yaml, an optional preset, an optional user file and overrides."""
    data = load_yaml(DEFAULT_YAML)
    if preset:
        p = PRESET_DIR / f"{preset}.yaml"
        if not p.exists():
            raise FileNotFoundError(f"unknown preset {preset!r}; have {sorted(x.stem for x in PRESET_DIR.glob('*.yaml'))}")
        deep_merge(data, load_yaml(p))
    if path:
        deep_merge(data, load_yaml(path))
    cfg = ConfigNode(data)
    apply_overrides(cfg, overrides)
    validate_config(cfg)
    return cfg


def redundant_settings(cfg: ConfigNode) -> tuple[int, int, int, int]:
    """(rollout_n, alg_rollout_n, entries_per_buffer, ready_entries_per_buffer).

    With redundant rollout enabled the PS over-provisions both the number of
    samples per prompt and the number of prompt groups per buffer
    (``psrl/workers/ps/ps_manager.py:78-110``).
    """
    p = cfg.psrl
    rr = p.rollout_coordination.redundant_rollout
    if rr.enable:
        return (
            int(rr.redundant_rollout_n),
            int(rr.alg_rollout_n),
            int(rr.redundant_global_batch_size),
            int(rr.alg_global_batch_size),
        )
    return int(p.rollout_n), int(p.rollout_n), int(p.staleness_buffer_entries), int(p.staleness_buffer_entries)


class ConfigError(ValueError):
    pass


def validate_config(cfg: ConfigNode) -> None:
    """Cross-group consistency checks (reference: ``psrl/utils/config.py:94``)."""
    p = cfg.psrl
    if p.staleness < 0:
        raise ConfigError("psrl.staleness must be >= 0")
    if p.staleness_buffer_entries <= 0:
        raise ConfigError("psrl.staleness_buffer_entries must be > 0")
    if p.rollout_n < 1:
        raise ConfigError("psrl.rollout_n must be >= 1")
    if p.ps_mode not in ("hbm", "cpu", "cpu_ref"):
        raise ConfigError(f"psrl.ps_mode={p.ps_mode!r} not supported (hbm|cpu|cpu_ref)")
    rr = p.rollout_coordination.redundant_rollout
    if rr.enable:
        if rr.redundant_rollout_n < rr.alg_rollout_n:
            raise ConfigError("redundant_rollout_n must be >= alg_rollout_n")
        if rr.redundant_global_batch_size < rr.alg_global_batch_size:
            raise ConfigError("redundant_global_batch_size must be >= alg_global_batch_size")
    adv = cfg.algorithm.adv_estimator
    if adv not in ("gae", "grpo", "reinforce_plus_plus", "gdpo", "optimal_token_baseline", "rloo"):
        raise ConfigError(f"unknown algorithm.adv_estimator {adv!r}")
    if adv == "gae" and not cfg.critic.enable:
        raise ConfigError("adv_estimator=gae needs critic.enable=true")
    if adv in ("grpo", "rloo", "gdpo") and p.rollout_n < 2 and not rr.enable:
        raise ConfigError(f"adv_estimator={adv} needs psrl.rollout_n >= 2 (group sampling)")
    mini = cfg.actor.ppo_mini_batch_size
    if mini <= 0 or p.staleness_buffer_entries % mini != 0:
        raise ConfigError("actor.ppo_mini_batch_size must divide psrl.staleness_buffer_entries")
    m = cfg.actor.megatron
    if cfg.actor.strategy == "megatron":
        if m.context_parallel_size > 1 and not cfg.model.use_remove_padding:
            raise ConfigError("context_parallel_size > 1 requires model.use_remove_padding")
    if cfg.actor.loss_agg_mode not in ("token-mean", "seq-mean-token-sum", "seq-mean-token-mean", "seq-mean-token-sum-norm"):
        raise ConfigError(f"unknown actor.loss_agg_mode {cfg.actor.loss_agg_mode!r}")
    fgo = p.fine_grain_overlap
    if fgo.granularity not in ("none", "mini_batch", "micro_batch"):
        raise ConfigError("fine_grain_overlap.granularity must be none|mini_batch|micro_batch")
    if fgo.overlap_scope not in ("recompute", "pre_step"):
        raise ConfigError("fine_grain_overlap.overlap_scope must be recompute|pre_step")
    sm = p.rollout_coordination.sync_and_mig_strategy.method
    if sm not in ("greedy", "status_based"):
        raise ConfigError("sync_and_mig_strategy.method must be greedy|status_based")
    rs = p.rollout_coordination.routing_strategy.method
    if rs not in ("random", "round_robin", "request_num_balance", "throughput_optimal",
                  "throughput_optimal_with_budget", "cache_aware", "cache_aware_v1"):
        raise ConfigError(f"unknown routing_strategy.method {rs!r}")
    alg = cfg.algorithm
    if alg.get("use_kl_in_reward"):
        if str(alg.get("kl_penalty", "kl")) not in ("kl", "k1", "abs", "mse", "k2", "low_var_kl", "k3"):
            raise ConfigError(f"unknown algorithm.kl_penalty {alg.kl_penalty!r}")
        kc = alg.get("kl_ctrl") or {}
        if str(kc.get("type", "fixed")) not in ("fixed", "adaptive"):
            raise ConfigError("algorithm.kl_ctrl.type must be fixed|adaptive")
        if str(kc.get("type", "fixed")) == "adaptive" and float(kc.get("target_kl", 0.1)) <= 0:
            raise ConfigError("algorithm.kl_ctrl.target_kl must be > 0")
    rc = alg.get("rollout_correction") or {}
    if rc.get("rollout_is") not in (None, "token", "sequence"):
        raise ConfigError("algorithm.rollout_correction.rollout_is must be null|token|sequence")
    if rc.get("rollout_rs") not in (None, "token", "sequence", "geometric"):
        raise ConfigError("algorithm.rollout_correction.rollout_rs must be null|token|sequence|geometric")
    d = cfg.data
    if d.kind in ("parquet", "jsonl", "files") and not d.get("train_files"):
        raise ConfigError(f"data.kind={d.kind} needs data.train_files")
    r = cfg.reward
    g = r.get("gen_rm") or {}
    if r.kind == "gen" and g.get("backend") == "http" and not g.get("url"):
        raise ConfigError("reward.gen_rm.backend=http needs reward.gen_rm.url")
    env = str(p.agentic_rl.get("env", "synthetic_tokens"))
    if env not in ("synthetic_tokens", "shell_env", "tool_env"):
        raise ConfigError(f"unknown psrl.agentic_rl.env {env!r}")


__all__ = [
    "ConfigNode",
    "ConfigError",
    "apply_overrides",
    "deep_merge",
    "load_config",
    "load_yaml",
    "parse_override",
    "redundant_settings",
    "validate_config",
]
