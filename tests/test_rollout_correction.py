"""Rollout correction between rollout-engine and trainer log-probs: truncated
importance weights (token / sequence) and rejection sampling (token /
sequence / geometric), their path into the packed micro-batch, and a
colocated training run with them enabled."""

import math

import torch

from psrl_b200.config import load_config
from psrl_b200.config.node import ConfigNode
from psrl_b200.trainer import algos
from psrl_b200.trainer.batch import Trajectory, build_micro_batch


def _traj(old, roll, rid=0, mask=None):
    n = len(old)
    return Trajectory(uid=0, request_id=rid, prompt_ids=[1, 2], response_ids=list(range(3, 3 + n)),
                      rollout_logprobs=list(roll), old_logprobs=list(old), response_mask=mask)


def _rc(**kw):
    base = {"rollout_is": None, "rollout_is_threshold": 2.0, "rollout_rs": None, "rollout_rs_threshold": 2.0,
            "rollout_rs_threshold_lower": None}
    base.update(kw)
    return ConfigNode(base)


def test_noop_when_disabled_or_identical():
    t = _traj([-1.0, -2.0], [-1.0, -2.0])
    assert algos.apply_rollout_correction(_rc(), [t]) == {}
    m = algos.apply_rollout_correction(_rc(rollout_is="token", rollout_rs="token"), [t])
    assert t.is_weights == [1.0, 1.0] and t.response_mask == [1, 1]
    assert m["rollout_corr/rs_masked_fraction"] == 0.0 and abs(m["rollout_corr/kl"]) < 1e-12


def test_token_is_weights_truncated():
    old, roll = [-1.0, -0.5, -3.0], [-1.2, -2.0, -2.9]
    t = _traj(old, roll)
    algos.apply_rollout_correction(_rc(rollout_is="token", rollout_is_threshold=2.0), [t])
    want = [min(math.exp(o - r), 2.0) for o, r in zip(old, roll)]
    assert all(abs(a - b) < 1e-9 for a, b in zip(t.is_weights, want))


def test_sequence_is_weight_is_the_truncated_product():
    old, roll = [-1.0, -0.9], [-1.1, -1.0]
    t = _traj(old, roll)
    algos.apply_rollout_correction(_rc(rollout_is="sequence", rollout_is_threshold=5.0), [t])
    w = math.exp(sum(o - r for o, r in zip(old, roll)))
    assert all(abs(x - w) < 1e-9 for x in t.is_weights)


def test_rejection_sampling_levels():
    old, roll = [-1.0, -0.1, -1.0], [-1.0, -1.5, -1.0]     # token 1 ratio e^1.4 > 2
    t = _traj(old, roll)
    algos.apply_rollout_correction(_rc(rollout_rs="token"), [t])
    assert t.response_mask == [1, 0, 1]
    t = _traj(old, roll)
    algos.apply_rollout_correction(_rc(rollout_rs="sequence"), [t])
    assert t.response_mask == [0, 0, 0]                     # product e^1.4 > 2
    t = _traj(old, roll)
    algos.apply_rollout_correction(_rc(rollout_rs="geometric"), [t])
    assert t.response_mask == [1, 1, 1]                     # geometric mean e^(1.4/3) < 2


def test_environment_tokens_stay_masked():
    t = _traj([-1.0, -1.0, -1.0], [-1.0, -1.0, -1.0], mask=[1, 0, 1])
    algos.apply_rollout_correction(_rc(rollout_rs="token", rollout_is="token"), [t])
    assert t.response_mask == [1, 0, 1] and t.is_weights[1] == 0.0


def test_weights_reach_the_micro_batch():
    a = _traj([-1.0, -0.5], [-1.2, -0.9], rid=0)
    b = _traj([-1.0], [-1.0], rid=1)
    algos.apply_rollout_correction(_rc(rollout_is="token"), [a])
    mb = build_micro_batch([a, b], [0, 1], "cpu")
    w = mb.extra["is_weights"]
    assert w.shape == mb.loss_mask.shape
    # a: 3 input tokens, labels of response start at index P-1 = 1
    torch.testing.assert_close(w[1:3], torch.tensor(a.is_weights, dtype=torch.float32))
    assert float(w[0]) == 1.0 and float(w[3:].sum()) == float(w[3:].numel())


def test_colocated_training_with_correction():
    torch.set_num_threads(2)
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "psrl.log_prob.enable_rollout_engine_log_prob=false", "algorithm.rollout_correction.rollout_is=sequence",
        "algorithm.rollout_correction.rollout_rs=token", "rollout.max_response_length=12"])
    t = RLTrainer(cfg)
    out = t.fit(2)
    t.stop_rollout()
    for m in out:
        assert 0.0 <= m["rollout_corr/rs_masked_fraction"] <= 1.0
        assert m["rollout_corr/is_weight_mean"] > 0.0
        assert math.isfinite(m["actor/pg_loss"])


def test_plan_counts_only_loss_tokens():
    from psrl_b200.trainer.actor import loss_tokens, plan_update
    a = _traj([-1.0] * 4, [-1.0] * 4, rid=0, mask=[1, 0, 0, 1])
    b = _traj([-1.0] * 3, [-1.0] * 3, rid=1)
    assert loss_tokens(a) == 2 and loss_tokens(b) == 3
    plans = plan_update([a, b], 2, 1)
    assert plans[0][0][1] == 5.0
