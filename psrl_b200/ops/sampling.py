"""Token sampling with log-probabilities (K9).

Plain temperature sampling (the RL rollout default: T=1, top_p=1, top_k=-1)
runs the fused Gumbel-max kernel (``csrc/logprob.cu::sample``): one pass over
the vocabulary yields the sampled token and its log-probability.  top-k /
top-p filtering (validation) uses a sort-based PyTorch path.
"""

from __future__ import annotations

import torch

from ._ext import ext


def sample_ref(logits, temps, seeds, streams, top_k=-1, top_p=1.0):
    z = logits.float()
    t = temps.float().clamp_min(1e-6)[:, None] if temps is not None else 1.0
    greedy = (temps <= 0) if temps is not None else torch.zeros(z.shape[0], dtype=torch.bool, device=z.device)
    z = z / t
    if top_k is not None and top_k > 0:
        kth = z.topk(min(top_k, z.shape[-1]), dim=-1).values[:, -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    if top_p is not None and top_p < 1.0:
        sz, si = z.sort(-1, descending=True)
        cp = sz.softmax(-1).cumsum(-1)
        drop = (cp - sz.softmax(-1)) > top_p
        sz = sz.masked_fill(drop, float("-inf"))
        z = torch.full_like(z, float("-inf")).scatter(-1, si, sz)
    logp = z.log_softmax(-1)
    gen = torch.Generator(device="cpu")
    toks = []
    for i in range(z.shape[0]):
        if bool(greedy[i]):
            toks.append(int(z[i].argmax()))
            continue
        stream = int(streams[i]) if streams is not None else 0
        gen.manual_seed((int(seeds[i]) if seeds is not None else 0) * 1_000_003 + stream)
        toks.append(int(torch.multinomial(logp[i].exp().cpu(), 1, generator=gen)))
    tok = torch.tensor(toks, dtype=torch.long, device=logits.device)
    return tok, logp.gather(-1, tok[:, None])[:, 0]


def sample(logits: torch.Tensor, temps: torch.Tensor | None = None, seeds: torch.Tensor | None = None,
           streams: torch.Tensor | None = None, top_k: int = -1, top_p: float = 1.0):
    """Returns (tokens int64 [B], logprobs fp32 [B]).

    ``temps`` fp32 [B] (<= 0: greedy), ``seeds`` int64 [B], ``streams`` int32 [B]
    (the position of the sampled token: randomness depends on (seed, position)).
    """
    if logits.is_cuda and (top_k is None or top_k <= 0) and (top_p is None or top_p >= 1.0):
        return ext().sample(logits, temps, seeds, streams)
    return sample_ref(logits, temps, seeds, streams, top_k, top_p)
