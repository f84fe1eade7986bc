"""Validation loop of the one-process trainer (test_freq): validation prompts
are generated with the current weights, scored, and do not leak into
training buffers."""

import pytest
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


_GPU_TINY = ["model.preset=tiny128", "model.dtype=bf16", "trainer.device=cuda", "rollout.cuda_graph=true",
             "data.kind=synthetic_tokens", "data.prompt_len_min=16", "data.prompt_len_max=64",
             "data.response_len_mu=3.0", "data.response_len_sigma=0.5", "data.response_len_cap=64",
             "reward.kind=bernoulli_hash", "rollout.ignore_eos=true"]


@pytest.mark.gpu
def test_validate_every_step_gpu():
    """The same validation loop on one GPU (CUDA-graph rollout engine, bf16)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=_GPU_TINY + ["trainer.test_freq=1", "++data.val_size=4"])
    t = RLTrainer(cfg)
    out = t.fit(2)
    assert all(m["val/num_samples"] == 4 * int(cfg.psrl.val_rollout_n) for m in out)
    assert all(0.0 <= m["val/score_mean"] <= 1.0 for m in out)
    assert all(m["num_trajectories"] == 32 for m in out)
    t.stop_rollout()


@pytest.mark.gpu
def test_ppo_with_critic_gpu():
    """PPO (GAE) with a critic on one GPU: value forward, critic update and
    actor update all finite."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import math

    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=_GPU_TINY + ["critic.enable=true",
                                                                      "algorithm.adv_estimator=gae"])
    t = RLTrainer(cfg)
    for _ in range(2):
        m = t.step()
        assert m["num_trajectories"] == 32
        assert math.isfinite(m["critic/vf_loss"]) and m["critic/vf_loss"] >= 0
        assert math.isfinite(m["actor/pg_loss"])
    t.stop_rollout()
