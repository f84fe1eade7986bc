"""Fused AdamW over flat fp32 master shards (part of K14).

One kernel per flat buffer updates master weights, both moments and writes
the bf16 working copy; the global gradient-norm clip coefficient is read from
device memory so the whole optimizer step has no host synchronisation.
"""

from __future__ import annotations

import torch

from ._ext import ext


def adamw_ref(p, g, m, v, p16, lr, b1, b2, eps, wd, step, gscale=1.0):
    g = g.float() * gscale
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    upd = (m / bc1) / ((v / bc2).sqrt() + eps)
    p.sub_(lr * (wd * p + upd))
    if p16 is not None:
        p16.copy_(p)


def adamw_(p, g, m, v, p16, lr, b1, b2, eps, wd, step, gscale_t: torch.Tensor | None = None, gscale: float = 1.0):
    if p.is_cuda:
        ext().adamw_(p, g, m, v, p16, lr, b1, b2, eps, wd, int(step), gscale_t, gscale)
    else:
        s = gscale * (float(gscale_t.item()) if gscale_t is not None else 1.0)
        adamw_ref(p, g, m, v, p16, lr, b1, b2, eps, wd, step, s)


class NormAccumulator:
    """Accumulates sum of squares of many tensors into a device scalar."""

    def __init__(self, device, max_ctas: int = 1024):
        self.device = torch.device(device)
        self.sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.partial = torch.empty(max_ctas, dtype=torch.float32, device=self.device)

    def reset(self):
        self.sq.zero_()

    def add(self, x: torch.Tensor):
        if x.is_cuda:
            ext().sqnorm_accumulate_(x.contiguous(), self.sq, self.partial)
        else:
            self.sq += x.float().pow(2).sum()

    def clip_coef(self, max_norm: float) -> tuple[torch.Tensor, torch.Tensor]:
        coef = torch.empty(1, dtype=torch.float32, device=self.device)
        norm = torch.empty(1, dtype=torch.float32, device=self.device)
        if self.device.type == "cuda":
            ext().clip_coef_(self.sq, float(max_norm), coef, norm)
        else:
            norm.copy_(self.sq.sqrt())
            coef.fill_(min(1.0, max_norm / (float(norm) + 1e-6)) if max_norm > 0 else 1.0)
        return coef, norm
