"""Fused LM-head log-probability (K8) and its backward.

``linear_logprob(h, W, labels)`` returns per-token log pi(label) and entropy
without ever materialising fp32 logits for the whole batch: logits are
produced one token chunk at a time (bf16 GEMM), reduced by a single-pass
online log-sum-exp kernel (``csrc/logprob.cu``), and recomputed in backward
where the softmax gradient is written in place before the two backward GEMMs.
"""

from __future__ import annotations

import torch

from ._ext import ext

DEFAULT_CHUNK = 16384
# inference log-probs through the fused tcgen05 kernel (csrc/gemm_sm100.cu) when shapes allow
USE_TCGEN05 = True


def linear_logprob_ref(h, W, labels, temperature: float = 1.0, want_entropy: bool = True):
    logits = (h.float() @ W.float().t()) / temperature
    logp = logits.log_softmax(-1)
    lp = logp.gather(-1, labels.clamp_min(0)[:, None].long())[:, 0]
    lp = torch.where(labels >= 0, lp, torch.zeros_like(lp))
    ent = -(logp.exp() * logp).sum(-1) if want_entropy else None
    return lp, ent


class _LinearLogprobFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, labels, temperature, chunk):
        T = h.shape[0]
        lps, ents, lses = [], [], []
        for s in range(0, T, chunk):
            logits = h[s: s + chunk] @ W.t()
            lp, ent, lse = ext().logprob_fwd(logits, labels[s: s + chunk], temperature, True)
            lps.append(lp)
            ents.append(ent)
            lses.append(lse)
        lp = torch.cat(lps) if len(lps) > 1 else lps[0]
        ent = torch.cat(ents) if len(ents) > 1 else ents[0]
        lse = torch.cat(lses) if len(lses) > 1 else lses[0]
        ctx.save_for_backward(h, W, labels, lse, ent)
        ctx.cfg = (temperature, chunk)
        return lp, ent

    @staticmethod
    def backward(ctx, glp, gent):
        h, W, labels, lse, ent = ctx.saved_tensors
        temperature, chunk = ctx.cfg
        T = h.shape[0]
        dh = torch.empty_like(h)
        dW = None
        for s in range(0, T, chunk):
            hc = h[s: s + chunk]
            logits = hc @ W.t()
            ext().logprob_bwd_(
                logits, labels[s: s + chunk], temperature,
                glp[s: s + chunk].contiguous().float() if glp is not None else None,
                gent[s: s + chunk].contiguous().float() if gent is not None else None,
                lse[s: s + chunk], ent[s: s + chunk])
            dh[s: s + chunk] = logits @ W
            part = logits.t() @ hc
            if T <= chunk:
                dW = part
            else:
                dW = part.float() if dW is None else dW.add_(part.float())
        return dh, dW.to(W.dtype), None, None, None


def linear_logprob(h: torch.Tensor, W: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0,
                   chunk: int = DEFAULT_CHUNK):
    """log-softmax(h W^T / T)[label] and entropy, both fp32 [T]."""
    labels = labels.long()
    if h.is_cuda and h.dtype == torch.bfloat16:
        needs_grad = torch.is_grad_enabled() and (h.requires_grad or W.requires_grad)
        from . import gemm as tc
        if not needs_grad and USE_TCGEN05 and tc.supported(h, W):
            # inference (old / reference log-probs): fused tcgen05 GEMM + log-sum-exp
            # epilogue, the [T, V] logits never leave tensor memory
            lp, ent, _ = tc.tc_linear_logprob(h, W, labels, temperature)
            return lp, ent
        # training: chunked logits in bf16, recomputed in backward (one consistent
        # rounding of the logits in both directions)
        return _LinearLogprobFn.apply(h, W, labels, float(temperature), int(chunk))
    return linear_logprob_ref(h, W, labels, temperature)


def logits_logprob(logits: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0):
    """Inference-only: (logprob, entropy) from precomputed logits rows."""
    if logits.is_cuda:
        lp, ent, _ = ext().logprob_fwd(logits, labels.long(), temperature, True)
        return lp, ent
    logp = (logits.float() / temperature).log_softmax(-1)
    lp = logp.gather(-1, labels.long().clamp_min(0)[:, None])[:, 0]
    return lp, -(logp.exp() * logp).sum(-1)
