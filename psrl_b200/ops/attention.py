"""Attention ops (K1, K2, K3).

* :func:`varlen_attention` — causal attention over a packed batch (training,
  remove-padding), autograd-enabled.  CUDA: forward on the tcgen05 / TMEM
  kernels ``attn_fwd_sm100`` / ``attn_bwd_sm100`` (``csrc/attn_sm100.cu``).
* :func:`paged_prefill_attention` — chunked prefill against the paged KV cache.
* :func:`paged_decode_attention` — one query token per sequence, split-KV.

The PyTorch implementations below are the numerical oracles and the CPU path.
"""

from __future__ import annotations

import math

import torch

from ._ext import ext


# --------------------------------------------------------------- references
def varlen_attention_ref(q, k, v, cu_seqlens, scale):
    """q [T, nq, d], k/v [T, nkv, d]; causal per sequence; fp32 math."""
    T, nq, d = q.shape
    nkv = k.shape[1]
    g = nq // nkv
    out = torch.empty(T, nq, d, dtype=q.dtype, device=q.device)
    cu = cu_seqlens.tolist()
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        if e <= s:
            continue
        qs = q[s:e].float().transpose(0, 1)                     # [nq, L, d]
        ks = k[s:e].float().transpose(0, 1).repeat_interleave(g, 0)
        vs = v[s:e].float().transpose(0, 1).repeat_interleave(g, 0)
        att = (qs @ ks.transpose(1, 2)) * scale
        L = e - s
        mask = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
        att = att.masked_fill(mask, float("-inf")).softmax(-1)
        out[s:e] = (att @ vs).transpose(0, 1).to(q.dtype)
    return out


def gather_paged_kv(k_cache, v_cache, block_table_row, length):
    bs = k_cache.shape[2]
    nblk = (length + bs - 1) // bs
    blocks = block_table_row[:nblk].long()
    k = k_cache[blocks].permute(0, 2, 1, 3).reshape(-1, k_cache.shape[1], k_cache.shape[3])[:length]
    v = v_cache[blocks].permute(0, 2, 1, 3).reshape(-1, v_cache.shape[1], v_cache.shape[3])[:length]
    return k, v


def paged_attention_ref(q, k_cache, v_cache, cu_q, kv_lens, block_table, scale):
    """Queries are the last q_len positions of each context (causal)."""
    T, nq, d = q.shape
    nkv = k_cache.shape[1]
    g = nq // nkv
    out = torch.empty_like(q)
    cu = cu_q.tolist()
    lens = kv_lens.tolist()
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        if e <= s:
            continue
        L = lens[i]
        k, v = gather_paged_kv(k_cache, v_cache, block_table[i], L)
        qs = q[s:e].float().transpose(0, 1)
        ks = k.float().transpose(0, 1).repeat_interleave(g, 0)
        vs = v.float().transpose(0, 1).repeat_interleave(g, 0)
        att = (qs @ ks.transpose(1, 2)) * scale            # [nq, ql, L]
        ql = e - s
        qpos = torch.arange(L - ql, L, device=q.device)[:, None]
        kpos = torch.arange(L, device=q.device)[None, :]
        att = att.masked_fill(kpos > qpos, float("-inf")).softmax(-1)
        out[s:e] = (att @ vs).transpose(0, 1).to(q.dtype)
    return out


# ----------------------------------------------------------------- autograd
class _VarlenAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cu_seqlens, max_seqlen, nq, nkv, d, scale):
        T = qkv.shape[0]
        o, lse = varlen_attention_fwd(qkv, cu_seqlens, max_seqlen, nq, nkv, scale, want_lse=True)
        o = o.view(T, nq, d)
        ctx.save_for_backward(qkv, o, lse, cu_seqlens)
        ctx.cfg = (max_seqlen, nq, nkv, d, scale)
        return o.view(T, nq * d)

    @staticmethod
    def backward(ctx, do):
        from .gemm import _err
        qkv, o, lse, cu = ctx.saved_tensors
        max_seqlen, nq, nkv, d, scale = ctx.cfg
        if qkv.stride(1) != 1 or qkv.stride(0) % 8 or qkv.data_ptr() % 16:
            qkv = qkv.contiguous()
        # tcgen05 backward (csrc/attn_sm100.cu): dK/dV per key tile and dQ per
        # query tile, written straight into one [T, (nq + 2 nkv) * d] gradient
        dqkv = ext().attn_bwd_sm100(qkv, o.reshape(qkv.shape[0], nq * d), do.contiguous(), lse, cu, max_seqlen,
                                    nq, nkv, scale, _err(qkv.device))
        return dqkv, None, None, None, None, None, None


def varlen_attention_fwd(qkv: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int, nq: int, nkv: int,
                         scale: float, want_lse: bool = True):
    """Forward of causal varlen attention on the tcgen05 kernel
    (``csrc/attn_sm100.cu``): ``qkv`` [T, (nq + 2 nkv) * 128] bf16 ->
    (o [T, nq * 128] bf16, lse [nq, T] fp32 natural log)."""
    from .gemm import _err
    if qkv.stride(1) != 1 or qkv.stride(0) % 8 or qkv.data_ptr() % 16:
        qkv = qkv.contiguous()
    return ext().attn_fwd_sm100(qkv, cu_seqlens, int(max_seqlen), int(nq), int(nkv), float(scale), bool(want_lse),
                                _err(qkv.device))


def varlen_attention(qkv: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int, nq: int, nkv: int, d: int,
                     scale: float | None = None) -> torch.Tensor:
    """Causal attention over a packed batch; ``qkv`` [T, (nq+2nkv)*d] -> [T, nq*d]."""
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if qkv.is_cuda and qkv.dtype == torch.bfloat16 and d == 128:
        if not torch.is_grad_enabled() or not qkv.requires_grad:
            return varlen_attention_fwd(qkv, cu_seqlens, max_seqlen, nq, nkv, scale, want_lse=False)[0]
        return _VarlenAttnFn.apply(qkv, cu_seqlens, int(max_seqlen), nq, nkv, d, scale)
    T = qkv.shape[0]
    q = qkv[:, : nq * d].view(T, nq, d)
    k = qkv[:, nq * d: (nq + nkv) * d].view(T, nkv, d)
    v = qkv[:, (nq + nkv) * d:].view(T, nkv, d)
    return _ref_autograd(q, k, v, cu_seqlens, scale).reshape(T, nq * d)


def _ref_autograd(q, k, v, cu_seqlens, scale):
    # differentiable reference (CPU training path)
    T, nq, d = q.shape
    nkv = k.shape[1]
    g = nq // nkv
    outs = []
    cu = cu_seqlens.tolist()
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        if e <= s:
            continue
        qs = q[s:e].transpose(0, 1)
        ks = k[s:e].transpose(0, 1).repeat_interleave(g, 0)
        vs = v[s:e].transpose(0, 1).repeat_interleave(g, 0)
        L = e - s
        mask = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
        att = ((qs @ ks.transpose(1, 2)) * scale).masked_fill(mask, float("-inf")).softmax(-1)
        outs.append((att @ vs).transpose(0, 1))
    return torch.cat(outs, 0) if outs else q.new_zeros(0, nq, d)


def paged_prefill_attention(q, k_cache, v_cache, cu_q, kv_lens, block_table, max_q_len, scale=None):
    """q [T, nq, d] (view ok); returns [T, nq, d]."""
    d = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if q.is_cuda and d == 128:
        return ext().attn_paged_prefill(q, k_cache, v_cache, cu_q, kv_lens, block_table, int(max_q_len), scale)
    return paged_attention_ref(q, k_cache, v_cache, cu_q, kv_lens, block_table, scale)


def decode_splits(batch: int, nkv: int, max_ctx: int) -> int:
    return int(ext().decode_num_splits(batch, nkv, max_ctx))


def paged_decode_attention(q, k_cache, v_cache, block_table, kv_lens, scale=None, splits: int | None = None,
                           scratch: torch.Tensor | None = None, stages: int = 0):
    """q [B, nq, d] -> [B, nq, d]; kv_lens include the current token."""
    d = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if q.is_cuda and d == 128:
        if splits is None:
            splits = decode_splits(q.shape[0], k_cache.shape[1], int(block_table.shape[1] * k_cache.shape[2]))
        if not (q.stride(2) == 1 and q.stride(1) == d and q.stride(0) % 8 == 0 and q.data_ptr() % 16 == 0):
            q = q.contiguous()
        return ext().attn_decode(q, k_cache, v_cache, block_table, kv_lens, scale, int(splits), scratch, int(stages))
    B = q.shape[0]
    cu = torch.arange(B + 1, dtype=torch.int32, device=q.device)
    return paged_attention_ref(q, k_cache, v_cache, cu, kv_lens, block_table, scale)


# ------------------------------------------- queries against separate keys
def attention_kv_ref(q, k, v, cu_q, cu_k, scale):
    """q [Tq, nq, d]; k / v [Tk, nkv, d]; sequence b's queries
    [cu_q[b], cu_q[b+1]) are the last of its key positions [cu_k[b], cu_k[b+1]),
    so query row p sees keys 0 .. p + Lk - Lq.  Differentiable, fp32 math."""
    Tq, nq, d = q.shape
    g = nq // k.shape[1]
    outs = []
    cq, ck = cu_q.tolist(), cu_k.tolist()
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], ck[b], ck[b + 1]
        Lq, Lk = qe - qs, ke - ks
        if Lq <= 0:
            continue
        qq = q[qs:qe].float().transpose(0, 1)
        kk = k[ks:ke].float().transpose(0, 1).repeat_interleave(g, 0)
        vv = v[ks:ke].float().transpose(0, 1).repeat_interleave(g, 0)
        rows = torch.arange(Lq, device=q.device)[:, None] + (Lk - Lq)
        mask = torch.arange(Lk, device=q.device)[None, :] > rows
        att = ((qq @ kk.transpose(1, 2)) * scale).masked_fill(mask, float("-inf")).softmax(-1)
        outs.append((att @ vv).transpose(0, 1).to(q.dtype))
    return torch.cat(outs, 0) if outs else q.new_zeros(0, nq, d)


class _AttnKVFn(torch.autograd.Function):
    """tcgen05 forward / backward of queries against separately stored keys
    (``attn_fwd_sm100_kv`` / ``attn_bwd_sm100_kv``)."""

    @staticmethod
    def forward(ctx, q, kv, cu_q, cu_k, max_q, max_k, nq, nkv, scale):
        from .gemm import _err
        o, lse = ext().attn_fwd_sm100_kv(q, kv, cu_q, cu_k, int(max_q), int(nq), int(nkv), float(scale), True,
                                         _err(q.device))
        ctx.save_for_backward(q, kv, o, lse, cu_q, cu_k)
        ctx.cfg = (max_q, max_k, nq, nkv, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        from .gemm import _err
        q, kv, o, lse, cu_q, cu_k = ctx.saved_tensors
        max_q, max_k, nq, nkv, scale = ctx.cfg
        dq, dkv = ext().attn_bwd_sm100_kv(q, kv, o, do.contiguous(), lse, cu_q, cu_k, int(max_q), int(max_k),
                                          int(nq), int(nkv), float(scale), _err(q.device))
        return dq, dkv, None, None, None, None, None, None, None


def attention_kv(q: torch.Tensor, kv: torch.Tensor, cu_q: torch.Tensor, cu_k: torch.Tensor, max_q: int, max_k: int,
                 nq: int, nkv: int, d: int, scale: float | None = None) -> torch.Tensor:
    """Causal attention of queries ``q`` [Tq, nq * d] against keys / values
    ``kv`` [Tk, 2 nkv * d] (k heads, then v heads) where each sequence's queries
    are the last ``Lq`` of its ``Lk >= Lq`` key positions; returns [Tq, nq * d].
    Context-parallel attention runs a rank's query chunks through this against
    the gathered key prefix."""
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    if q.is_cuda and q.dtype == torch.bfloat16 and d == 128:
        if q.stride(1) != 1 or q.stride(0) % 8 or q.data_ptr() % 16:
            q = q.contiguous()
        return _AttnKVFn.apply(q, kv.contiguous(), cu_q, cu_k, int(max_q), int(max_k), nq, nkv, scale)
    Tq, Tk = q.shape[0], kv.shape[0]
    o = attention_kv_ref(q.reshape(Tq, -1)[:, : nq * d].reshape(Tq, nq, d), kv[:, : nkv * d].reshape(Tk, nkv, d),
                         kv[:, nkv * d:].reshape(Tk, nkv, d), cu_q, cu_k, scale)
    return o.reshape(Tq, nq * d)
