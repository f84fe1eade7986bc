"""Validation loop of the one-process trainer (test_freq): validation prompts
are generated with the current weights, scored, and do not leak into
training buffers."""

import torch


def test_validate_every_step_cpu():
    torch.set_num_threads(2)
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["trainer.test_freq=1", "++data.val_size=4",
                                                         "rollout.max_response_length=12"])
    t = RLTrainer(cfg)
    out = t.fit(2)
    assert all("val/score_mean" in m for m in out)
    assert all(m["val/num_samples"] == 4 * int(cfg.psrl.val_rollout_n) for m in out)
    assert all(0.0 <= m["val/score_mean"] <= 1.0 for m in out)
    # validation uids never enter a training buffer
    assert all(m["num_trajectories"] == 32 for m in out)
    r = t.validate(3)
    assert r["val/num_samples"] == 3 * int(cfg.psrl.val_rollout_n)
    t.stop_rollout()
