"""Rotary embeddings (K5), rotate-half convention, theta configurable (1e6 for
Qwen2.5/Qwen3).  CUDA: ``csrc/rope.cu`` (in place on the fused qkv activation,
optionally fused with the paged KV-cache write)."""

from __future__ import annotations

import math

import torch

from ._ext import ext

_TABLES: dict = {}


def inv_frequencies(spec, dim: int) -> torch.Tensor:
    """float64 [dim/2] rotary frequencies.  ``spec`` is the base, or
    ``(base, (key, value), ...)`` with a scaling rule (``ModelArgs.rope_spec``):

    * ``linear``: every frequency divided by ``factor`` (positions stretched);
    * ``llama3``: wavelengths shorter than ``original / high_freq_factor`` kept,
      longer than ``original / low_freq_factor`` divided by ``factor``, and a
      linear blend (in ``original / wavelength``) between the two bands.
    """
    if isinstance(spec, tuple):
        theta, opts = float(spec[0]), dict(spec[1:])
    else:
        theta, opts = float(spec), {}
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    kind = opts.get("rope_type", "default")
    if kind == "linear":
        inv = inv / float(opts["factor"])
    elif kind == "llama3":
        factor = float(opts["factor"])
        lo, hi = float(opts.get("low_freq_factor", 1.0)), float(opts.get("high_freq_factor", 4.0))
        orig = float(opts.get("original_max_position_embeddings", 8192))
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        blended = (1.0 - smooth) * inv / factor + smooth * inv
        inv = torch.where(wavelen < orig / hi, inv, torch.where(wavelen > orig / lo, inv / factor, blended))
    elif kind != "default":
        raise NotImplementedError(f"RoPE scaling {kind!r}")
    return inv


def rope_tables(theta, dim: int, max_pos: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin tables of shape [max_pos, dim/2] computed in float64;
    ``theta`` is a base or a ``ModelArgs.rope_spec``."""
    key = (theta if isinstance(theta, tuple) else float(theta), int(dim), str(device))
    have = _TABLES.get(key)
    if have is not None and have[0].shape[0] >= max_pos:
        return have
    n = max(int(max_pos), 4096)
    inv = inv_frequencies(theta, dim)
    ang = torch.arange(n, dtype=torch.float64)[:, None] * inv[None, :]
    tabs = (ang.cos().float().to(device), ang.sin().float().to(device))
    _TABLES[key] = tabs
    return tabs


def apply_rope_ref(x: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, inverse=False):
    """x: [T, heads, d]."""
    c = cos[positions.long()][:, None, :]
    s = sin[positions.long()][:, None, :]
    if inverse:
        s = -s
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def rope_qkv_(qkv: torch.Tensor, positions: torch.Tensor, nq: int, nkv: int, d: int, theta: float,
              inverse: bool = False, k_cache=None, v_cache=None, slots=None) -> torch.Tensor:
    """Rotate the q and k heads of ``qkv`` [T, (nq+2nkv)*d] in place."""
    T = qkv.shape[0]
    if T == 0:
        return qkv
    maxp = int(positions.max().item()) + 1 if not qkv.is_cuda else 0
    if qkv.is_cuda:
        cos, sin = rope_tables(theta, d, 65536, qkv.device)
        ext().rope_(qkv, positions.int() if positions.dtype != torch.int32 else positions, cos, sin, nq, nkv, d,
                    inverse, k_cache, v_cache, slots)
        return qkv
    cos, sin = rope_tables(theta, d, maxp, qkv.device)
    q = qkv[:, : nq * d].view(T, nq, d)
    k = qkv[:, nq * d: (nq + nkv) * d].view(T, nkv, d)
    q.copy_(apply_rope_ref(q, positions, cos, sin, inverse))
    k.copy_(apply_rope_ref(k, positions, cos, sin, inverse))
    if k_cache is not None:
        v = qkv[:, (nq + nkv) * d:].view(T, nkv, d)
        write_kv_cache_ref(k, v, k_cache, v_cache, slots)
    return qkv


def write_kv_cache_ref(k, v, k_cache, v_cache, slots):
    """Cache layout [blocks, nkv, block_size, d]; slots < 0 are skipped."""
    bs = k_cache.shape[2]
    sl = slots.long()
    ok = sl >= 0
    blk, off = sl[ok] // bs, sl[ok] % bs
    k_cache[blk, :, off] = k[ok].to(k_cache.dtype)
    v_cache[blk, :, off] = v[ok].to(v_cache.dtype)


class _RopeFn(torch.autograd.Function):
    """Training RoPE on a fused qkv activation (out of place for autograd)."""

    @staticmethod
    def forward(ctx, qkv, positions, nq, nkv, d, theta):
        out = qkv.clone()
        rope_qkv_(out, positions, nq, nkv, d, theta)
        ctx.save_for_backward(positions)
        ctx.cfg = (nq, nkv, d, theta)
        return out

    @staticmethod
    def backward(ctx, g):
        (positions,) = ctx.saved_tensors
        nq, nkv, d, theta = ctx.cfg
        g = g.contiguous().clone()
        rope_qkv_(g, positions, nq, nkv, d, theta, inverse=True)
        return g, None, None, None, None, None


def rope_qkv(qkv, positions, nq, nkv, d, theta):
    return _RopeFn.apply(qkv, positions, nq, nkv, d, theta)
