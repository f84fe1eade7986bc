"""In-reward KL: the fixed and adaptive coefficient controllers, the per-token
reward rows, the advantage estimators on KL-shaped rewards, and the
sharded (two gloo ranks) recomputation against the single-process one."""

import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from psrl_b200.config import load_config
from psrl_b200.trainer import algos
from psrl_b200.trainer.batch import Trajectory
from psrl_b200.trainer.driver import compute_batch_advantages


def _trajs(seed=0, n_groups=4, per_group=4):
    g = torch.Generator().manual_seed(seed)
    out, rid = [], 0
    for u in range(n_groups):
        for _ in range(per_group):
            n = int(torch.randint(2, 9, (1,), generator=g))
            old = (-torch.rand(n, generator=g) * 2).tolist()
            ref = (torch.tensor(old) + torch.randn(n, generator=g) * 0.3).tolist()
            out.append(Trajectory(uid=u, request_id=rid, prompt_ids=[1, 2, 3], response_ids=list(range(5, 5 + n)),
                                  rollout_logprobs=old, reward=float(torch.rand(1, generator=g)), old_logprobs=old,
                                  ref_logprobs=ref))
            rid += 1
    return out


def test_fixed_controller_is_constant():
    c = algos.FixedKLController(0.05)
    c.update(10.0, 100)
    assert c.value == 0.05


def test_adaptive_controller_proportional_step():
    c = algos.AdaptiveKLController(0.1, target_kl=0.2, horizon=1000)
    c.update(0.3, n_steps=50)                # error 0.5 clipped to 0.2
    assert math.isclose(c.value, 0.1 * (1 + 0.2 * 50 / 1000))
    c2 = algos.AdaptiveKLController(0.1, target_kl=0.2, horizon=1000)
    c2.update(0.18, n_steps=100)             # error -0.1
    assert math.isclose(c2.value, 0.1 * (1 - 0.1 * 100 / 1000))


def test_controller_from_config():
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["algorithm.kl_ctrl.type=adaptive",
                                                         "algorithm.kl_ctrl.kl_coef=0.02"])
    c = algos.kl_controller(cfg.algorithm)
    assert isinstance(c, algos.AdaptiveKLController) and c.value == 0.02


@pytest.mark.parametrize("kind", ["kl", "abs", "mse", "low_var_kl"])
def test_token_rewards_match_definition(kind):
    trajs = _trajs()
    ctrl = algos.FixedKLController(0.1)
    m = algos.apply_kl_in_reward(trajs, ctrl, kind)
    kls = []
    for t in trajs:
        kld = algos.kl_penalty(torch.tensor(t.old_logprobs), torch.tensor(t.ref_logprobs), kind)
        want = -0.1 * kld
        want[-1] += t.reward
        torch.testing.assert_close(torch.tensor(t.token_rewards), want, rtol=1e-6, atol=1e-6)
        kls.append(float(kld.mean()))
    assert math.isclose(m["actor/reward_kl_penalty"], sum(kls) / len(kls), rel_tol=1e-5)
    assert m["actor/reward_kl_penalty_coeff"] == 0.1


def test_env_tokens_carry_no_kl():
    t = _trajs(n_groups=1, per_group=1)[0]
    n = t.response_len
    t.response_mask = [1] * (n - 2) + [0, 1]
    algos.apply_kl_in_reward([t], algos.FixedKLController(1.0), "kl")
    assert t.token_rewards[n - 2] == 0.0


def test_grpo_scores_are_kl_shaped_sums():
    cfg = load_config(preset="cpu_tiny_grpo")
    trajs = _trajs(1)
    ctrl = algos.FixedKLController(0.2)
    compute_batch_advantages(cfg, trajs, ctrl)
    scores = torch.tensor([sum(t.token_rewards) for t in trajs])
    want = algos.grpo_outcome_advantage(scores, [t.uid for t in trajs], True)
    torch.testing.assert_close(torch.tensor([t.advantage for t in trajs]), want)


def test_reinforce_pp_uses_token_rewards():
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["algorithm.adv_estimator=reinforce_plus_plus"])
    trajs = _trajs(2)
    compute_batch_advantages(cfg, trajs, algos.FixedKLController(0.5))
    L = max(t.response_len for t in trajs)
    rew, mask = torch.zeros(len(trajs), L), torch.zeros(len(trajs), L)
    for i, t in enumerate(trajs):
        rew[i, :t.response_len] = torch.tensor(t.token_rewards)
        mask[i, :t.response_len] = 1
    want = algos.reinforce_pp_returns(rew, mask, 1.0)
    for i, t in enumerate(trajs):
        torch.testing.assert_close(torch.tensor(t.token_advantages), want[i, :t.response_len], rtol=1e-5, atol=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, est, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"algorithm.adv_estimator={est}"])
    trajs = _trajs(3)
    mine = [t for i, t in enumerate(trajs) if (i * 7 + 3) % world == rank]     # groups split across ranks
    ctrl = algos.AdaptiveKLController(0.3, 0.05, 100)
    m = algos.shard_advantages(cfg, mine, dist.group.WORLD, ctrl)
    q.put({"rank": rank, "coef": ctrl.value, "kl": m["actor/reward_kl_penalty"],
           "adv": {t.request_id: (t.advantage, t.token_advantages) for t in mine}})
    dist.destroy_process_group()


@pytest.mark.parametrize("est", ["grpo", "reinforce_plus_plus"])
def test_sharded_advantages_match_single_process(est):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, est, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
    assert [p.exitcode for p in procs] == [0, 0]
    res = [q.get(timeout=5) for _ in range(2)]
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[f"algorithm.adv_estimator={est}"])
    trajs = _trajs(3)
    ctrl = algos.AdaptiveKLController(0.3, 0.05, 100)
    m = compute_batch_advantages(cfg, trajs, ctrl)
    for r in res:
        assert math.isclose(r["coef"], ctrl.value, rel_tol=1e-9)
        assert math.isclose(r["kl"], m["actor/reward_kl_penalty"], rel_tol=1e-6)
        for rid, (a, ta) in r["adv"].items():
            t = trajs[rid]
            if est == "grpo":
                assert math.isclose(a, t.advantage, rel_tol=1e-5, abs_tol=1e-6)
            else:
                torch.testing.assert_close(torch.tensor(ta), torch.tensor(t.token_advantages), rtol=1e-4, atol=1e-5)


def test_colocated_trainer_applies_in_reward_kl():
    torch.set_num_threads(2)
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["algorithm.use_kl_in_reward=true",
                                                         "algorithm.kl_ctrl.type=adaptive",
                                                         "rollout.max_response_length=12"])
    t = RLTrainer(cfg)
    out = t.fit(2)
    t.stop_rollout()
    assert all("actor/reward_kl_penalty" in m for m in out)
    assert out[0]["actor/reward_kl_penalty_coeff"] == 0.001
    assert out[1]["actor/reward_kl_penalty_coeff"] != 0.001          # adaptive update after step 0
