"""Per-step perf metrics under the reference's names."""

import torch


def test_perf_metrics_formula():
    from psrl_b200.config import load_config
    from psrl_b200.models import PRESETS
    from psrl_b200.models.qwen import flops_per_token
    from psrl_b200.trainer.perf import perf_metrics
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["++trainer.peak_tflops=1000"])
    a = PRESETS["tiny"]
    m = perf_metrics(cfg, a, tokens=8000, num_trajectories=8, step_s=2.0, train_s=1.0, n_gpus=4, n_train_gpus=2)
    assert m["perf/throughput"] == 8000 / 2.0 / 4
    assert abs(m["perf/mfu/actor"] - 3 * flops_per_token(a, 1000) * 8000 / (1.0 * 2 * 1e15)) < 1e-12
    assert m["perf/total_num_tokens"] == 8000 and m["perf/time_per_step"] == 2.0


def test_trainer_step_reports_perf():
    torch.set_num_threads(2)
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    t = RLTrainer(load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12"]))
    m = t.step()
    t.stop_rollout()
    assert m["perf/throughput"] > 0 and m["perf/mfu/actor"] > 0
    assert m["perf/total_num_tokens"] == m["trained_tokens"]


def test_profiler_window_and_turn_records(tmp_path):
    """trainer.profile_steps writes a torch-profiler trace for those steps only;
    trainer.turn_records_path gets one JSON line per finished request."""
    import json
    import os
    torch.set_num_threads(2)
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    turns = str(tmp_path / "turns.jsonl")
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "rollout.max_response_length=12", "++trainer.profile_steps=[1]", f"++trainer.profile_dir={tmp_path}/tr",
        f"++trainer.turn_records_path={turns}"])
    t = RLTrainer(cfg)
    out = t.fit(2)
    t.stop_rollout()
    assert "profile/trace" not in out[0] and os.path.exists(out[1]["profile/trace"])
    with open(turns) as fh:
        recs = [json.loads(line) for line in fh]
    assert len(recs) >= 32 and all("turns" in r for r in recs)


def test_engine_stats_recorded(tmp_path):
    """trainer.engine_stats_path: one engine snapshot per step (one-process
    trainer), readable back through StatsRecorder."""
    torch.set_num_threads(2)
    from psrl_b200.config import load_config
    from psrl_b200.rollout.stats import StatsRecorder
    from psrl_b200.trainer import RLTrainer
    path = str(tmp_path / "stats.jsonl")
    t = RLTrainer(load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12",
                                                                 f"++trainer.engine_stats_path={path}"]))
    t.fit(2)
    t.stop_rollout()
    recs = StatsRecorder(path).read()
    assert len(recs) == 2 and all("kv_usage" in r and "num_running" in r for r in recs)
