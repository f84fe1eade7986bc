"""Trajectory records and packed (remove-padding) micro-batches.

A trajectory is one sampled response to one prompt.  For training, a
trajectory of prompt length P and response length R contributes P + R - 1
input tokens (the last token is only a label).  Micro-batches are packed up to
a token budget (``ppo_max_token_len_per_gpu``, "dynamic batch size") with a
first-fit-decreasing assignment; DP ranks receive token-balanced shares
(``_balance_batch`` in the reference trainer).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from ..utils import transfer


@dataclass
class Trajectory:
    uid: int                      # prompt group id (GRPO group key)
    request_id: int
    prompt_ids: list
    response_ids: list
    rollout_logprobs: list
    reward: float = 0.0
    versions: list = field(default_factory=list)
    version_tag: int = 0
    advantage: float = 0.0        # outcome-level advantage (filled by the driver)
    token_advantages: list | None = None  # token-level (GAE / REINFORCE++)
    returns: list | None = None
    old_values: list | None = None
    ref_logprobs: list | None = None
    old_logprobs: list | None = None
    response_mask: list | None = None   # multi-turn: 0 on environment tokens
    token_rewards: list | None = None   # per-token rewards when the in-reward KL term is applied
    is_weights: list | None = None      # rollout-correction importance weights per response token
    meta: dict = field(default_factory=dict)

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.response_ids) - 1

    @property
    def response_len(self) -> int:
        return len(self.response_ids)


@dataclass
class MicroBatch:
    input_ids: torch.Tensor       # [T] int64
    positions: torch.Tensor       # [T] int32
    cu_seqlens: torch.Tensor      # [B+1] int32
    max_seqlen: int
    labels: torch.Tensor          # [T] int64 (-1 where no label)
    loss_mask: torch.Tensor       # [T] float (1 on response-token labels)
    old_logprobs: torch.Tensor    # [T] float
    advantages: torch.Tensor      # [T] float
    seq_ids: torch.Tensor         # [T] int64 (index of the trajectory within the micro-batch)
    traj_index: list              # indices into the source trajectory list
    extra: dict = field(default_factory=dict)

    @property
    def num_tokens(self) -> int:
        return int(self.input_ids.numel())


def balance_across_ranks(trajs: list[Trajectory], world: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of trajectories to ranks by token count."""
    order = sorted(range(len(trajs)), key=lambda i: -trajs[i].num_tokens)
    loads = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = int(np.argmin(loads))
        parts[r].append(i)
        loads[r] += trajs[i].num_tokens
    return parts


def pack_micro_batches(idx: list[int], trajs: list[Trajectory], max_tokens: int) -> list[list[int]]:
    """First-fit-decreasing bins of at most ``max_tokens`` tokens (a longer
    single trajectory gets a bin of its own)."""
    order = sorted(idx, key=lambda i: -trajs[i].num_tokens)
    bins: list[list[int]] = []
    loads: list[int] = []
    for i in order:
        n = trajs[i].num_tokens
        for b in range(len(bins)):
            if loads[b] + n <= max_tokens:
                bins[b].append(i)
                loads[b] += n
                break
        else:
            bins.append([i])
            loads.append(n)
    return bins


def build_micro_batch(trajs: list[Trajectory], idx: list[int], device, field_old: str = "old_logprobs") -> MicroBatch:
    ids, pos, labels, mask, old, adv, seq, isw = [], [], [], [], [], [], [], []
    cu = [0]
    any_isw = any(trajs[i].is_weights is not None for i in idx)
    for j, i in enumerate(idx):
        t = trajs[i]
        toks = list(t.prompt_ids) + list(t.response_ids)
        n = len(toks) - 1
        P = len(t.prompt_ids)
        ids.append(np.asarray(toks[:-1], dtype=np.int64))
        pos.append(np.arange(n, dtype=np.int32))
        lab = np.asarray(toks[1:], dtype=np.int64)
        labels.append(lab)
        m = np.zeros(n, dtype=np.float32)
        m[P - 1:] = 1.0 if t.response_mask is None else np.asarray(t.response_mask, dtype=np.float32)
        mask.append(m)
        o = np.zeros(n, dtype=np.float32)
        src = getattr(t, field_old) if getattr(t, field_old) is not None else t.rollout_logprobs
        o[P - 1:] = np.asarray(src, dtype=np.float32)
        old.append(o)
        a = np.zeros(n, dtype=np.float32)
        if t.token_advantages is not None:
            a[P - 1:] = np.asarray(t.token_advantages, dtype=np.float32)
        else:
            a[P - 1:] = t.advantage
        adv.append(a)
        if any_isw:
            w = np.ones(n, dtype=np.float32)
            if t.is_weights is not None:
                w[P - 1:] = np.asarray(t.is_weights, dtype=np.float32)
            isw.append(w)
        seq.append(np.full(n, j, dtype=np.int64))
        cu.append(cu[-1] + n)

    on_gpu = torch.device(device).type == "cuda"

    def cat(xs, dtype):
        t = torch.from_numpy(np.concatenate(xs)).to(dtype)
        if on_gpu:
            t = t.pin_memory()
        return t.to(device=device, non_blocking=True)

    lens = [cu[k + 1] - cu[k] for k in range(len(idx))]
    transfer.h2d(cu[-1] * 40 + 4 * len(cu))
    return MicroBatch(
        input_ids=cat(ids, torch.long), positions=cat(pos, torch.int32),
        cu_seqlens=torch.tensor(cu, dtype=torch.int32).to(device), max_seqlen=max(lens) if lens else 0,
        labels=cat(labels, torch.long), loss_mask=cat(mask, torch.float32), old_logprobs=cat(old, torch.float32),
        advantages=cat(adv, torch.float32), seq_ids=cat(seq, torch.long), traj_index=list(idx),
        extra={"is_weights": cat(isw, torch.float32)} if any_isw else {})


def response_slices(mb: MicroBatch, trajs: list[Trajectory]):
    """(trajectory index, slice into the packed token axis covering its response labels)."""
    out = []
    cu = mb.cu_seqlens.tolist()
    for j, i in enumerate(mb.traj_index):
        P = len(trajs[i].prompt_ids)
        out.append((i, slice(cu[j] + P - 1, cu[j + 1])))
    return out
