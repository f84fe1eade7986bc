"""Token-level estimators (GAE, REINFORCE++) on multi-turn responses.

Environment observation tokens inside a response carry ``response_mask`` 0.
They must take no TD step and no discount step, and must stay out of the
whitening statistics.  So a trajectory with observation spans gives the same
advantages on its action tokens as the same trajectory with those spans cut
out.
"""

import torch

from psrl_b200.config import load_config
from psrl_b200.trainer import algos
from psrl_b200.trainer.batch import Trajectory


def _pair(seed: int):
    """(multi-turn trajectory with observation spans, same trajectory with the
    spans removed, indices of the action tokens in the first)."""
    g = torch.Generator().manual_seed(seed)
    turns = [int(x) for x in torch.randint(2, 6, (3,), generator=g)]
    obs = [int(x) for x in torch.randint(1, 4, (2,), generator=g)]
    mask, keep = [], []
    for i, n in enumerate(turns):
        keep += list(range(len(mask), len(mask) + n))
        mask += [1] * n
        if i < len(obs):
            mask += [0] * obs[i]
    L = len(mask)
    values = torch.randn(L, generator=g).tolist()
    reward = float(torch.rand(1, generator=g))
    full = Trajectory(uid=seed, request_id=seed, prompt_ids=[1, 2], response_ids=list(range(L)),
                      rollout_logprobs=[0.0] * L, reward=reward, response_mask=mask, old_values=values)
    cut = Trajectory(uid=seed, request_id=seed, prompt_ids=[1, 2], response_ids=[full.response_ids[i] for i in keep],
                     rollout_logprobs=[0.0] * len(keep), reward=reward, old_values=[values[i] for i in keep])
    return full, cut, keep


def _rows(trajs):
    L = max(t.response_len for t in trajs)
    rew, vals, mask = torch.zeros(len(trajs), L), torch.zeros(len(trajs), L), torch.zeros(len(trajs), L)
    for i, t in enumerate(trajs):
        n = t.response_len
        mask[i, :n] = algos.response_mask_row(t)
        rew[i, :n] = torch.tensor(algos.token_reward_row(t))
        vals[i, :n] = torch.tensor(t.old_values[:n])
    return rew, vals, mask


def test_gae_skips_observation_tokens():
    pairs = [_pair(s) for s in range(4)]
    fulls, cuts = [p[0] for p in pairs], [p[1] for p in pairs]
    r1, v1, m1 = _rows(fulls)
    r2, v2, m2 = _rows(cuts)
    for gamma, lam in ((1.0, 0.95), (0.9, 0.8)):
        a1, ret1 = algos.gae_advantage(r1, v1, m1, gamma, lam)
        a2, ret2 = algos.gae_advantage(r2, v2, m2, gamma, lam)
        for i, (_, cut, keep) in enumerate(pairs):
            n = cut.response_len
            assert torch.allclose(a1[i, keep], a2[i, :n], atol=1e-5)
            assert torch.allclose(ret1[i, keep], ret2[i, :n], atol=1e-5)


def test_reinforce_pp_skips_observation_tokens():
    pairs = [_pair(10 + s) for s in range(4)]
    r1, _, m1 = _rows([p[0] for p in pairs])
    r2, _, m2 = _rows([p[1] for p in pairs])
    a1 = algos.reinforce_pp_returns(r1, m1, 0.97)
    a2 = algos.reinforce_pp_returns(r2, m2, 0.97)
    for i, (_, cut, keep) in enumerate(pairs):
        assert torch.allclose(a1[i, keep], a2[i, :cut.response_len], atol=1e-5)


def test_global_whitening_uses_response_mask():
    cfg = load_config(overrides=["algorithm.adv_estimator=gae", "critic.enable=true", "algorithm.gamma=1.0",
                                 "algorithm.lam=0.95"])
    pairs = [_pair(20 + s) for s in range(3)]
    fulls, cuts = [p[0] for p in pairs], [p[1] for p in pairs]
    algos.gae_with_global_whitening(cfg, fulls)
    algos.gae_with_global_whitening(cfg, cuts)
    for full, cut, keep in pairs:
        got = torch.tensor(full.token_advantages)[keep]
        assert torch.allclose(got, torch.tensor(cut.token_advantages), atol=1e-5)
        # observation tokens carry no advantage into the loss
        obs = [j for j in range(full.response_len) if j not in keep]
        assert all(full.token_advantages[j] == 0.0 for j in obs)
