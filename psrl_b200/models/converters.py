"""Tensor-parallel layouts of the fused parameters (C18 converters).

The trainer stores full fused tensors; a TP-``t`` rollout rank ``r`` holds

* ``attn.qkv``  — its query heads and its KV heads: rows
  ``[q_r | k_r | v_r]`` (column parallel; when nkv < t the KV heads are
  replicated across the ranks that share them);
* ``attn.o``    — the columns of its query heads (row parallel);
* ``mlp.gate_up`` — its slice of the gate rows followed by the same slice of
  the up rows (column parallel, so SwiGLU stays local);
* ``mlp.down``  — the matching input columns (row parallel);
* embeddings / LM head — vocabulary rows split (vocab parallel);
* norms / biases of row-parallel layers — replicated.

``tp_slices(name, shape, args, r, t)`` returns the (dim, start, length) pieces
of the full tensor that make rank ``r``'s local tensor, in order; the weight
sync turns them into copy segments.  MoE experts of a tensor-parallel trainer
are split along their SwiGLU width (ETP: ``experts_w13`` like ``gate_up`` for
every expert, ``experts_w2`` like ``down``), and so is a shared expert.
"""

from __future__ import annotations

from .config import ModelArgs


def tp_slices(name: str, shape: tuple, a: ModelArgs, r: int, t: int) -> list[tuple[int, int, int]]:
    if t == 1:
        return [(0, 0, shape[0])]
    d = a.head_dim
    if name.endswith("attn.qkv.weight") or name.endswith("attn.qkv.bias"):
        if a.num_heads % t:
            raise ValueError("num_heads must divide by tp")
        qh = a.num_heads // t
        if a.num_kv_heads >= t:
            if a.num_kv_heads % t:
                raise ValueError("num_kv_heads must divide by tp")
            kvh, kv0 = a.num_kv_heads // t, r * (a.num_kv_heads // t)
        else:
            kvh, kv0 = 1, r * a.num_kv_heads // t      # replicated KV head
        q = (0, r * qh * d, qh * d)
        k = (0, a.q_size + kv0 * d, kvh * d)
        v = (0, a.q_size + a.kv_size + kv0 * d, kvh * d)
        return [q, k, v]
    if name.endswith("attn.o.weight"):
        qh = a.num_heads // t
        return [(1, r * qh * d, qh * d)]
    if name.endswith("mlp.gate_up.weight"):
        inter = shape[0] // 2
        per = inter // t
        return [(0, r * per, per), (0, inter + r * per, per)]
    if name.endswith("mlp.down.weight"):
        per = shape[1] // t
        return [(1, r * per, per)]
    if name in ("embed.weight", "lm_head.weight"):
        per = -(-shape[0] // t)
        lo = r * per
        return [(0, lo, max(0, min(per, shape[0] - lo)))]
    if name.endswith("experts_w13"):
        # [E, 2 I, h]: the same gate / up split as gate_up, for every expert
        inter = shape[1] // 2
        per = inter // t
        return [(1, r * per, per), (1, inter + r * per, per)]
    if name.endswith("experts_w2"):
        per = shape[2] // t
        return [(2, r * per, per)]
    if name.endswith("mlp.shared_gate_up.weight"):
        inter = shape[0] // 2
        per = inter // t
        return [(0, r * per, per), (0, inter + r * per, per)]
    if name.endswith("mlp.shared_down.weight"):
        per = shape[1] // t
        return [(1, r * per, per)]
    return [(0, 0, shape[0])]      # replicated


def local_shape(name: str, shape: tuple, a: ModelArgs, r: int, t: int) -> tuple:
    sl = tp_slices(name, shape, a, r, t)
    dim = sl[0][0]
    n = sum(x[2] for x in sl)
    s = list(shape)
    s[dim] = n
    return tuple(s)


def shard_tensor(full, name: str, a: ModelArgs, r: int, t: int):
    import torch
    slices = tp_slices(name, tuple(full.shape), a, r, t)
    parts = [full.narrow(dim, start, length) for dim, start, length in slices]
    return torch.cat(parts, dim=slices[0][0]) if len(parts) > 1 else parts[0].contiguous()


def copy_segments_for(name: str, shape: tuple, itemsize: int, a: ModelArgs, r: int, t: int,
                      src_base: int, dst_base: int) -> list[tuple[int, int, int]]:
    """(src_byte_off, dst_byte_off, nbytes) runs that build rank r's local tensor
    from the full row-major tensor stored at ``src_base`` into ``dst_base``."""
    out = []
    lshape = local_shape(name, shape, a, r, t)
    acc = 0
    for dim, start, length in tp_slices(name, shape, a, r, t):
        inner = itemsize
        for x in shape[dim + 1:]:
            inner *= x
        outer = 1
        for x in shape[:dim]:
            outer *= x
        # one run per index of the leading dimensions
        for i in range(outer):
            out.append((src_base + (i * shape[dim] + start) * inner, dst_base + (i * lshape[dim] + acc) * inner,
                        length * inner))
        acc += length
    return out
