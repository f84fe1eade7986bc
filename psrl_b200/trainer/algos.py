"""RL algorithm math: advantage estimators, policy/value losses, KL penalties.

Behaviour follows the estimators the reference selects through veRL's
``core_algos`` (reference glue: ``psrl/trainer/ppo/utils.py:133-308``):

* ``gae`` — generalised advantage estimation over response tokens;
* ``grpo`` — outcome reward normalised within the prompt group (``uid`` /
  ``parent_id``), optionally divided by the group std;
* ``rloo`` — leave-one-out group baseline;
* ``reinforce_plus_plus`` — discounted returns whitened over the batch;
* ``gdpo`` — each reward component is group-normalised separately, then summed
  and re-normalised over the batch;
* ``optimal_token_baseline`` — per-position baseline weighted by squared
  sequence-length-normalised log-prob gradients (approximated by token counts);
* multi-trajectory GRPO broadcasts the final session's advantage to every
  output of that session (``compute_advantage_for_multi_trajectories``).

Losses: PPO clipped surrogate with asymmetric ("clip-higher") ranges and the
dual-clip lower bound ``clip_ratio_c``; aggregation modes ``token-mean``,
``seq-mean-token-sum``, ``seq-mean-token-mean``, ``seq-mean-token-sum-norm``;
clipped value loss; KL estimators k1/k2/k3(low_var_kl)/abs.
"""

from __future__ import annotations

from collections import defaultdict

import torch

# ------------------------------------------------------------------ helpers


def masked_mean(x: torch.Tensor, mask: torch.Tensor, dim=None, eps: float = 1e-8) -> torch.Tensor:
    m = mask.to(x.dtype)
    if dim is None:
        return (x * m).sum() / (m.sum() + eps)
    return (x * m).sum(dim) / (m.sum(dim) + eps)


def masked_whiten(x: torch.Tensor, mask: torch.Tensor, shift_mean: bool = True, eps: float = 1e-8) -> torch.Tensor:
    mean = masked_mean(x, mask)
    var = masked_mean((x - mean) ** 2, mask)
    out = (x - mean) * torch.rsqrt(var + eps)
    if not shift_mean:
        out = out + mean
    return out * mask


def group_indices(uids) -> dict:
    groups: dict = defaultdict(list)
    for i, u in enumerate(uids):
        groups[u].append(i)
    return groups


# --------------------------------------------------------------- advantages


def grpo_outcome_advantage(scores: torch.Tensor, uids, norm_by_std: bool = True, eps: float = 1e-6) -> torch.Tensor:
    """scores [N] (one scalar per trajectory) -> advantages [N]."""
    adv = torch.zeros_like(scores, dtype=torch.float32)
    for idx in group_indices(uids).values():
        s = scores[idx].float()
        if len(idx) == 1:
            mean, std = torch.zeros(()), torch.ones(())
        else:
            mean, std = s.mean(), s.std(unbiased=True)
        a = s - mean
        if norm_by_std:
            a = a / (std + eps)
        adv[idx] = a
    return adv


def rloo_advantage(scores: torch.Tensor, uids) -> torch.Tensor:
    adv = torch.zeros_like(scores, dtype=torch.float32)
    for idx in group_indices(uids).values():
        s = scores[idx].float()
        n = len(idx)
        adv[idx] = s - (s.sum() - s) / (n - 1) if n > 1 else s * 0
    return adv


def gdpo_advantage(score_components: torch.Tensor, uids, eps: float = 1e-6) -> torch.Tensor:
    """score_components [N, K]: group-normalise each component, sum, batch-whiten."""
    N, K = score_components.shape
    total = torch.zeros(N, dtype=torch.float32)
    for k in range(K):
        total += grpo_outcome_advantage(score_components[:, k], uids, True, eps)
    return (total - total.mean()) / (total.std(unbiased=False) + eps) if N > 1 else total


def reinforce_pp_returns(token_rewards: torch.Tensor, mask: torch.Tensor, gamma: float = 1.0) -> torch.Tensor:
    """token_rewards/mask [N, L] -> whitened discounted returns [N, L]."""
    return masked_whiten(discounted_returns(token_rewards, mask, gamma), mask)


def discounted_returns(token_rewards: torch.Tensor, mask: torch.Tensor, gamma: float = 1.0) -> torch.Tensor:
    """Discounted reward-to-go over the action tokens only: a token with
    mask 0 (padding, or an environment observation inside a multi-turn
    response) takes no discount step and passes the running return through
    unchanged, so a trajectory gives the same returns on its action tokens
    with or without its observation spans."""
    ret = torch.zeros_like(token_rewards, dtype=torch.float32)
    run = torch.zeros(token_rewards.shape[0], dtype=torch.float32)
    for t in reversed(range(token_rewards.shape[1])):
        m = mask[:, t].float()
        run = m * (token_rewards[:, t].float() + gamma * run) + (1.0 - m) * run
        ret[:, t] = run
    return ret


def gae_advantage(token_rewards: torch.Tensor, values: torch.Tensor, mask: torch.Tensor, gamma: float, lam: float,
                  whiten: bool = True):
    """[N, L] tensors -> (advantages [N, L] (whitened over the batch unless
    ``whiten`` is False), returns [N, L]).

    Tokens with mask 0 (padding, environment observations of a multi-turn
    response) take no TD step: the next value and the running lambda-return
    are carried across them unchanged, as veRL's
    ``compute_gae_advantage_return`` does with its response mask
    (``psrl/trainer/ppo/utils.py:167-172`` passes it)."""
    N, L = token_rewards.shape
    adv = torch.zeros(N, L, dtype=torch.float32)
    last = torch.zeros(N, dtype=torch.float32)
    nextv = torch.zeros(N, dtype=torch.float32)
    for t in reversed(range(L)):
        m = mask[:, t].float()
        delta = token_rewards[:, t].float() + gamma * nextv - values[:, t].float()
        last = m * (delta + gamma * lam * last) + (1.0 - m) * last
        adv[:, t] = last
        nextv = m * values[:, t].float() + (1.0 - m) * nextv
    returns = adv + values.float()
    return (masked_whiten(adv, mask) if whiten else adv * mask), returns * mask


def optimal_token_baseline_advantage(scores: torch.Tensor, uids, lengths: torch.Tensor, eps: float = 1e-6):
    """Group baseline weighted by 1/length (shorter trajectories' gradients are
    larger per token), normalised by the weighted group std."""
    adv = torch.zeros_like(scores, dtype=torch.float32)
    for idx in group_indices(uids).values():
        s = scores[idx].float()
        w = 1.0 / lengths[idx].float().clamp_min(1)
        b = (w * s).sum() / (w.sum() + eps)
        d = s - b
        sd = ((w * d * d).sum() / (w.sum() + eps)).sqrt()
        adv[idx] = d / (sd + eps) if len(idx) > 1 else d * 0
    return adv


def broadcast_session_advantage(adv: torch.Tensor, session_ids, is_final) -> torch.Tensor:
    """Multi-trajectory GRPO: every output of a session takes the final output's advantage."""
    out = adv.clone()
    final = {}
    for i, (sid, fin) in enumerate(zip(session_ids, is_final)):
        if fin:
            final[sid] = adv[i]
    for i, sid in enumerate(session_ids):
        if sid in final:
            out[i] = final[sid]
    return out


# -------------------------------------------------------------------- KL


def kl_penalty(logp: torch.Tensor, ref_logp: torch.Tensor, kind: str = "low_var_kl") -> torch.Tensor:
    d = logp - ref_logp
    if kind in ("kl", "k1"):
        return d
    if kind == "abs":
        return d.abs()
    if kind in ("mse", "k2"):
        return 0.5 * d * d
    if kind in ("low_var_kl", "k3"):
        r = torch.exp(-d.clamp(-20, 20))
        return (r - 1 + d).clamp(-10, 10)
    raise ValueError(f"unknown kl kind {kind!r}")


# -------------------------------------------------------------------- loss


def agg_loss(loss_mat: torch.Tensor, mask: torch.Tensor, mode: str, seq_ids: torch.Tensor | None = None,
             num_seqs: int | None = None, global_tokens: float | None = None, max_len: int | None = None):
    """Aggregate per-token losses of a packed micro-batch.

    ``global_tokens`` (token-mean) / ``num_seqs`` (seq-mean-*) are the counts over
    the whole mini-batch, so summing micro-batch losses gives the mini-batch mean.
    """
    m = mask.to(loss_mat.dtype)
    if mode == "token-mean":
        denom = global_tokens if global_tokens is not None else m.sum().clamp_min(1)
        return (loss_mat * m).sum() / denom
    assert seq_ids is not None, "seq-mean modes need per-token sequence ids"
    nseq = int(seq_ids.max().item()) + 1 if seq_ids.numel() else 0
    per_sum = torch.zeros(nseq, dtype=loss_mat.dtype, device=loss_mat.device).index_add_(0, seq_ids, loss_mat * m)
    per_cnt = torch.zeros(nseq, dtype=loss_mat.dtype, device=loss_mat.device).index_add_(0, seq_ids, m)
    denom = num_seqs if num_seqs is not None else max(nseq, 1)
    if mode == "seq-mean-token-sum":
        return per_sum.sum() / denom
    if mode == "seq-mean-token-mean":
        return (per_sum / per_cnt.clamp_min(1)).sum() / denom
    if mode == "seq-mean-token-sum-norm":
        return per_sum.sum() / (denom * (max_len or 1))
    raise ValueError(f"unknown loss_agg_mode {mode!r}")


def ppo_policy_loss(logp: torch.Tensor, old_logp: torch.Tensor, adv: torch.Tensor, mask: torch.Tensor,
                    clip_low: float, clip_high: float, clip_c: float | None, agg_mode: str = "token-mean",
                    tis_weight: torch.Tensor | None = None, **agg_kw):
    """Clipped surrogate (DAPO clip-higher + dual clip).  Returns (loss, metrics)."""
    neg_approx_kl = (logp - old_logp).clamp(-20.0, 20.0)
    ratio = torch.exp(neg_approx_kl)
    pg1 = -adv * ratio
    pg2 = -adv * ratio.clamp(1.0 - clip_low, 1.0 + clip_high)
    clipped = torch.maximum(pg1, pg2)
    if clip_c is not None and clip_c > 1.0:
        pg3 = -adv * clip_c
        dual = torch.minimum(pg3, clipped)
        pg = torch.where(adv < 0, dual, clipped)
    else:
        pg = clipped
    if tis_weight is not None:
        pg = pg * tis_weight
    loss = agg_loss(pg, mask, agg_mode, **agg_kw)
    with torch.no_grad():  # device tensors: no host sync inside the micro-batch loop
        m = mask.float()
        n = m.sum().clamp_min(1)
        metrics = {
            "pg_clipfrac": ((pg2 > pg1).float() * m).sum() / n,
            "ppo_kl": (-neg_approx_kl * m).sum() / n,
        }
        if clip_c:
            metrics["pg_clipfrac_lower"] = (((-adv * clip_c) < clipped).float() * (adv < 0).float() * m).sum() / n
    return loss, metrics


def value_loss(values: torch.Tensor, old_values: torch.Tensor, returns: torch.Tensor, mask: torch.Tensor,
               cliprange: float, agg_mode: str = "token-mean", **agg_kw):
    vclip = old_values + (values - old_values).clamp(-cliprange, cliprange)
    l1 = (values - returns) ** 2
    l2 = (vclip - returns) ** 2
    loss = 0.5 * agg_loss(torch.maximum(l1, l2), mask, agg_mode, **agg_kw)
    with torch.no_grad():
        m = mask.float()
        frac = ((l2 > l1).float() * m).sum() / m.sum().clamp_min(1)
    return loss, {"vf_clipfrac": frac}


def truncated_is_weight(old_logp: torch.Tensor, rollout_logp: torch.Tensor, cap: float) -> torch.Tensor:
    """TIS: min(pi_old / pi_rollout, cap) per token (rollout correction)."""
    return torch.exp((old_logp - rollout_logp).clamp(max=20.0)).clamp(max=cap).detach()


def compute_advantages(estimator: str, *, scores: torch.Tensor, uids, gamma: float = 1.0, lam: float = 1.0,
                       norm_by_std: bool = True, token_rewards=None, values=None, mask=None, lengths=None,
                       score_components=None):
    """Dispatch on ``algorithm.adv_estimator``; outcome estimators return [N],
    token-level ones return [N, L]."""
    if estimator == "grpo":
        return grpo_outcome_advantage(scores, uids, norm_by_std)
    if estimator == "rloo":
        return rloo_advantage(scores, uids)
    if estimator == "gdpo":
        comps = score_components if score_components is not None else scores[:, None]
        return gdpo_advantage(comps, uids)
    if estimator == "optimal_token_baseline":
        return optimal_token_baseline_advantage(scores, uids, lengths)
    if estimator == "reinforce_plus_plus":
        return reinforce_pp_returns(token_rewards, mask, gamma)
    if estimator == "gae":
        return gae_advantage(token_rewards, values, mask, gamma, lam)
    raise ValueError(f"unknown adv_estimator {estimator!r}")


# ------------------------------------------------------- rollout correction


def apply_rollout_correction(rc, trajs) -> dict:
    """Off-policy correction between the rollout engine's log-probs and the
    trainer's old-policy log-probs, per trajectory (after ``old_logprobs``
    are known; a no-op when both are the same numbers).

    ``rc.rollout_is`` (``token`` | ``sequence``): importance weights
    ``pi_old / pi_rollout`` (per token, or the product over the sequence),
    truncated at ``rollout_is_threshold``; stored as ``is_weights`` and
    multiplied into the policy loss.  ``rc.rollout_rs`` (``token`` |
    ``sequence`` | ``geometric``): rejection sampling, which zeroes
    ``response_mask`` on tokens (or whole sequences) whose ratio (token,
    sequence product, or per-token geometric mean) leaves
    ``[rollout_rs_threshold_lower, rollout_rs_threshold]`` (lower bound
    defaults to the reciprocal of the upper).

    Reference: ``psrl/trainer/ppo/ray_trainer.py:2843-2856`` (veRL's
    ``compute_rollout_correction_and_add_to_batch``).
    """
    level = rc.get("rollout_is", None)
    rs = rc.get("rollout_rs", None)
    if not level and not rs:
        return {}
    thr = float(rc.get("rollout_is_threshold", 2.0))
    hi = float(rc.get("rollout_rs_threshold", 2.0))
    lo = rc.get("rollout_rs_threshold_lower", None)
    lo = 1.0 / hi if lo is None else float(lo)
    kept = total = 0.0
    kl_sum = w_sum = 0.0
    n_seq = 0
    for t in trajs:
        ln = t.response_len
        if ln == 0 or t.old_logprobs is None:
            continue
        old = torch.tensor(t.old_logprobs[:ln], dtype=torch.float64)
        roll = torch.tensor(t.rollout_logprobs[:ln], dtype=torch.float64)
        m = (torch.tensor(t.response_mask[:ln], dtype=torch.float64) if t.response_mask is not None
             else torch.ones(ln, dtype=torch.float64))
        lr = (old - roll).clamp(-20.0, 20.0) * m
        cnt = float(m.sum())
        total += cnt
        kl_sum += float((-lr).sum() / max(cnt, 1.0))
        n_seq += 1
        if rs:
            if rs == "token":
                r = torch.exp(lr)
                keep = ((r >= lo) & (r <= hi)).double()
            else:
                agg = lr.sum() if rs == "sequence" else lr.sum() / max(cnt, 1.0)
                r = float(torch.exp(agg.clamp(-20.0, 20.0)))
                keep = torch.full((ln,), 1.0 if lo <= r <= hi else 0.0, dtype=torch.float64)
            m = m * keep
            t.response_mask = [int(x) for x in m.tolist()]
        kept += float(m.sum())
        if level:
            if level == "token":
                w = torch.exp(lr).clamp(max=thr)
            elif level == "sequence":
                w = torch.full((ln,), float(torch.exp(lr.sum().clamp(-20.0, 20.0)).clamp(max=thr)),
                               dtype=torch.float64)
            else:
                raise ValueError(f"unknown rollout_is level {level!r}")
            t.is_weights = (w * m).tolist()
            w_sum += float((w * m).sum() / max(float(m.sum()), 1.0))
    out = {"rollout_corr/kl": kl_sum / max(n_seq, 1)}
    if rs:
        out["rollout_corr/rs_masked_fraction"] = 1.0 - kept / max(total, 1.0)
    if level:
        out["rollout_corr/is_weight_mean"] = w_sum / max(n_seq, 1)
    return out


# --------------------------------------------------------- in-reward KL


class FixedKLController:
    """Constant in-reward KL coefficient (``algorithm.kl_ctrl.type=fixed``)."""

    def __init__(self, kl_coef: float):
        self.value = float(kl_coef)

    def update(self, current_kl: float, n_steps: int) -> None:
        pass


class AdaptiveKLController:
    """Proportional controller of Ziegler et al. 2019 ("Fine-Tuning Language
    Models from Human Preferences", section 2.2): the coefficient moves toward
    the value that keeps the measured KL at ``target_kl``, by at most 20 %
    of ``n_steps / horizon`` per update."""

    def __init__(self, init_kl_coef: float, target_kl: float, horizon: int):
        self.value = float(init_kl_coef)
        self.target = float(target_kl)
        self.horizon = int(horizon)

    def update(self, current_kl: float, n_steps: int) -> None:
        err = min(max(float(current_kl) / self.target - 1.0, -0.2), 0.2)
        self.value *= 1.0 + err * float(n_steps) / self.horizon


def kl_controller(alg_cfg):
    """The in-reward KL controller ``algorithm.kl_ctrl`` names (reference
    config ``psrl/trainer/config/ppo_trainer.yaml`` ``algorithm.kl_ctrl``)."""
    kc = alg_cfg.get("kl_ctrl", None) or {}
    kind = str(kc.get("type", "fixed"))
    coef = float(kc.get("kl_coef", alg_cfg.get("kl_coef", 0.001)))
    if kind == "fixed":
        return FixedKLController(coef)
    if kind == "adaptive":
        return AdaptiveKLController(coef, float(kc.get("target_kl", 0.1)), int(kc.get("horizon", 10000)))
    raise ValueError(f"unknown kl_ctrl.type {kind!r}")


def token_reward_row(t) -> list:
    """Per-response-token rewards of one trajectory: the in-reward KL rewards
    when they were applied, else the outcome reward on the last token."""
    if getattr(t, "token_rewards", None) is not None:
        return list(t.token_rewards)
    row = [0.0] * t.response_len
    if row:
        row[-1] = float(t.reward)
    return row


def trajectory_score(t) -> float:
    """Sequence score an outcome estimator normalises: the sum of the
    per-token rewards (the outcome reward when no KL term was applied)."""
    if getattr(t, "token_rewards", None) is not None:
        return float(sum(t.token_rewards))
    return float(t.reward)


def apply_kl_in_reward(trajs, ctrl, kind: str = "kl", group=None, replicas: int = 1) -> dict:
    """Per-token rewards ``score·[last] - beta·KL(old || ref)`` on every
    trajectory (``token_rewards``), then one controller update with the batch
    KL (each trajectory's masked token mean, averaged over trajectories).

    With ``group`` the KL statistic is summed over its ranks (one all-reduce
    of two numbers), so every rank applies the same coefficient update.
    When each trajectory sits on ``replicas`` ranks of the group (tensor-
    parallel replicas of one data-parallel share), both sums scale alike and
    the mean is unchanged; ``n_steps`` divides the count by ``replicas``.

    Reference: ``psrl/trainer/ppo/ray_trainer.py:2834-2842`` (veRL's
    ``apply_kl_penalty`` with ``kl_ctrl_in_reward``).
    """
    import torch.distributed as dist
    beta = float(ctrl.value)
    kl_sum, n = 0.0, 0
    for t in trajs:
        ln = t.response_len
        if ln == 0:
            t.token_rewards = []
            continue
        old = t.old_logprobs if t.old_logprobs is not None else t.rollout_logprobs
        lp = torch.tensor(old[:ln], dtype=torch.float32)
        ref = torch.tensor(t.ref_logprobs[:ln], dtype=torch.float32)
        m = torch.tensor(t.response_mask[:ln], dtype=torch.float32) if t.response_mask is not None else torch.ones(ln)
        kld = kl_penalty(lp, ref, kind) * m
        row = (-beta * kld)
        row[ln - 1] += float(t.reward)
        t.token_rewards = row.tolist()
        kl_sum += float(kld.sum() / m.sum().clamp_min(1.0))
        n += 1
    st = torch.tensor([kl_sum, float(n)], dtype=torch.float64)
    if group is not None and dist.is_initialized():
        dist.all_reduce(st, group=group)
    current = float(st[0] / st[1].clamp_min(1.0))
    ctrl.update(current, n_steps=int(round(float(st[1]) / max(1, int(replicas)))))
    return {"actor/reward_kl_penalty": current, "actor/reward_kl_penalty_coeff": beta}


def score_components(trajs):
    """[N, K] reward components from the ``gdpo`` reward loop (stored in
    ``meta["reward_extra"]["components"]``), or None when any trajectory
    lacks them or their counts differ."""
    rows = [((t.meta or {}).get("reward_extra") or {}).get("components") for t in trajs]
    if not rows or any(r is None for r in rows) or len({len(r) for r in rows}) != 1:
        return None
    return torch.tensor(rows, dtype=torch.float32)


def outcome_advantages_global(cfg, trajs, group=None) -> None:
    """Outcome estimator over the trajectories of every rank in ``group``:
    each rank contributes ``(request_id, uid, score, length)`` of its own
    trajectories (one all-gather of small records), duplicates (replicas that
    hold the same share) are dropped by ``request_id``, the estimator runs on
    the whole set, and each rank keeps its own trajectories' advantages."""
    import torch.distributed as dist
    comps = score_components(trajs)
    mine = [(int(t.request_id), t.uid, trajectory_score(t), t.response_len,
             comps[i].tolist() if comps is not None else None) for i, t in enumerate(trajs)]
    recs = [mine]
    if group is not None and dist.is_initialized():
        recs = [None] * dist.get_world_size(group)
        dist.all_gather_object(recs, mine, group=group)
    seen: dict = {}
    for part in recs:
        for r in part:
            seen.setdefault(r[0], r)
    allr = [seen[k] for k in sorted(seen)]
    if not allr:
        return
    comp_rows = [r[4] for r in allr]
    comps = (torch.tensor(comp_rows, dtype=torch.float32)
             if all(c is not None for c in comp_rows) and len({len(c) for c in comp_rows}) == 1 else None)
    adv = compute_advantages(cfg.algorithm.adv_estimator, scores=torch.tensor([r[2] for r in allr]),
                             uids=[r[1] for r in allr], norm_by_std=bool(cfg.algorithm.norm_adv_by_std_in_grpo),
                             lengths=torch.tensor([r[3] for r in allr]), score_components=comps)
    pos = {r[0]: i for i, r in enumerate(allr)}
    for t in trajs:
        t.advantage = float(adv[pos[int(t.request_id)]])
        t.token_advantages = None


def shard_advantages(cfg, trajs, group=None, kl_ctrl=None, replicas: int = 1, critic: bool = False) -> dict:
    """Advantages on one rank's share of a batch that is spread over
    ``group`` (the multi-GPU placements, where the control plane already
    filled the outcome advantages from the trajectory rewards).

    In-reward KL (``kl_ctrl``) changes every trajectory's reward, so outcome
    estimators are recomputed over the whole batch and token-level ones
    (REINFORCE++) are recomputed with global whitening; with a critic GAE
    always runs here on the rank's values."""
    out: dict = {}
    if kl_ctrl is not None:
        out.update(apply_kl_in_reward(trajs, kl_ctrl, str(cfg.algorithm.get("kl_penalty", "kl")), group, replicas))
    token_level = cfg.algorithm.adv_estimator in ("gae", "reinforce_plus_plus")
    if critic or (kl_ctrl is not None and token_level):
        gae_with_global_whitening(cfg, trajs, group)
    elif kl_ctrl is not None:
        outcome_advantages_global(cfg, trajs, group)
    return out


def response_mask_row(t) -> torch.Tensor:
    """[response_len] float mask of the tokens the policy produced: the
    trajectory's ``response_mask`` when set (0 on environment observations
    of a multi-turn response), else all ones."""
    n = t.response_len
    if t.response_mask is None:
        return torch.ones(n)
    m = torch.zeros(n)
    src = torch.tensor(t.response_mask[:n], dtype=torch.float32)
    m[: src.numel()] = src
    return m


def gae_with_global_whitening(cfg, trajs, group=None) -> None:
    """GAE (``old_values`` set) or, with no critic, REINFORCE++ returns on
    this rank's trajectories, whitened with the mean and variance of all
    ranks' response tokens in ``group`` (one all-reduce of three numbers);
    fills ``token_advantages`` and ``returns``.  Per-token rewards come from
    ``token_reward_row`` (in-reward KL when applied)."""
    import torch.distributed as dist
    L = max((t.response_len for t in trajs), default=1)
    N = len(trajs)
    rew, vals, mask = torch.zeros(N, L), torch.zeros(N, L), torch.zeros(N, L)
    use_values = all(t.old_values is not None for t in trajs)
    for i, t in enumerate(trajs):
        n = t.response_len
        mask[i, :n] = response_mask_row(t)
        rew[i, :n] = torch.tensor(token_reward_row(t), dtype=torch.float32)
        if use_values:
            vals[i, :n] = torch.tensor(t.old_values[:n])
    if use_values:
        adv, ret = gae_advantage(rew, vals, mask, float(cfg.algorithm.gamma), float(cfg.algorithm.lam),
                                 whiten=False)
    else:
        ret = discounted_returns(rew, mask, float(cfg.algorithm.gamma))
        adv = ret * mask
    st = torch.tensor([float((adv * mask).sum()), float((adv * adv * mask).sum()), float(mask.sum())],
                      dtype=torch.float64)
    if group is not None and dist.is_initialized():
        dist.all_reduce(st, group=group)
    mean = st[0] / st[2].clamp_min(1)
    var = st[1] / st[2].clamp_min(1) - mean * mean
    adv = ((adv - float(mean)) * float(torch.rsqrt(var.clamp_min(0) + 1e-8))) * mask
    if not use_values:
        ret = adv
    for i, t in enumerate(trajs):
        n = t.response_len
        t.token_advantages = adv[i, :n].tolist()
        t.returns = ret[i, :n].tolist()
