"""Fused LM-head log-probability (K8) and its backward.

``linear_logprob(h, W, labels)`` returns per-token log pi(label) and entropy
without materialising logits in the forward (fused tcgen05 GEMM + log-sum-exp
epilogue); the backward recomputes bf16 logits one token chunk at a time on
the tcgen05 GEMM, writes the softmax gradient in place (``csrc/logprob.cu``)
and runs the two backward GEMMs on tcgen05 as well.
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
    """Training LM head on the tcgen05 kernels.

    Forward: the fused GEMM + log-sum-exp kernel (``csrc/gemm_sm100.cu``
    EPI_LSE) over all T rows at once; no logits reach memory.  Backward, per
    chunk of rows: logits recomputed by the paired tcgen05 GEMM (bf16), their
    log-sum-exp and entropy re-derived from those same bf16 logits (so the
    softmax gradient sums to zero over the vocabulary), the softmax gradient
    written in place, then dH = dZ W and dW += dZ^T H as tcgen05 GEMMs reading
    dZ and H in place (MN-major), dW accumulated in fp32 by TMA reduce-add."""

    @staticmethod
    def forward(ctx, h, W, labels, temperature, chunk):
        from . import gemm as tc
        lp, ent, _ = tc.tc_linear_logprob(h, W, labels, temperature)
        ctx.save_for_backward(h, W, labels)
        ctx.cfg = (temperature, chunk)
        return lp, ent

    @staticmethod
    def backward(ctx, glp, gent):
        from .linear import matmul_nt
        h, W, labels = ctx.saved_tensors
        temperature, chunk = ctx.cfg
        T = h.shape[0]
        dh = torch.empty_like(h)
        dW32 = torch.zeros(W.shape, dtype=torch.float32, device=W.device)
        for s in range(0, T, chunk):
            hc = h[s: s + chunk]
            lab = labels[s: s + chunk]
            logits = matmul_nt(hc, W)
            _, ent_c, lse_c = ext().logprob_fwd(logits, lab, temperature, True)
            ext().logprob_bwd_(
                logits, lab, temperature,
                glp[s: s + chunk].contiguous().float() if glp is not None else None,
                gent[s: s + chunk].contiguous().float() if gent is not None else None,
                lse_c, ent_c)
            dh[s: s + chunk] = matmul_nt(logits, W, b_mn=True)
            matmul_nt(logits, hc, a_mn=True, b_mn=True, out=dW32)
            del logits
        return dh, dW32.to(W.dtype), None, None, None


def linear_logprob(h: torch.Tensor, W: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0,
                   chunk: int = DEFAULT_CHUNK):
    """log-softmax(h W^T / T)[label] and entropy, both fp32 [T]."""
    labels = labels.long()
    if h.is_cuda and h.dtype == torch.bfloat16:
        needs_grad = torch.is_grad_enabled() and (h.requires_grad or W.requires_grad)
        from . import gemm as tc
        if not (USE_TCGEN05 and tc.supported(h, W)):
            raise RuntimeError(f"tcgen05 LM head: unsupported operands h{tuple(h.shape)} W{tuple(W.shape)}")
        if not needs_grad:
            # inference (old / reference log-probs): fused tcgen05 GEMM + log-sum-exp
            # epilogue, the [T, V] logits never leave tensor memory
            lp, ent, _ = tc.tc_linear_logprob(h, W, labels, temperature)
            return lp, ent
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
