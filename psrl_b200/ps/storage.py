"""PS storage planning (C10): which PS worker holds what, how a new PS group is
initialised from one loaded copy, and the train→gen dtype cast.

* :class:`PSStoragePlan` assigns the flat parameter range evenly to ``n`` storage
  shards (one per trainer rank in ``ps_mode=hbm``).
* :class:`BinaryTreeBroadcastPlan` initialises ``n`` stores from store 0 in
  ``ceil(log2 n)`` rounds: in round r every store that already has the data
  sends to the store ``2^r`` positions further (reference
  ``psrl/workers/ps/broadcast.py:63-160``).
* :func:`cast_train_to_gen` produces the generation copy: bf16 (identity) or
  fp8-e4m3 with one fp32 scale per 128x128 block (the block-scaled format the
  rollout uses when serving fp8).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class PSStoragePlan:
    total: int
    n_shards: int

    def shard_range(self, i: int) -> tuple[int, int]:
        per = math.ceil(self.total / self.n_shards)
        lo = min(self.total, i * per)
        return lo, min(self.total, lo + per)

    def owner_of(self, offset: int) -> int:
        per = math.ceil(self.total / self.n_shards)
        return min(self.n_shards - 1, offset // per)


class BinaryTreeBroadcastPlan:
    def __init__(self, n: int, root: int = 0):
        self.n = int(n)
        self.root = int(root)

    def rounds(self) -> list[list[tuple[int, int]]]:
        """List of rounds; each round is a list of (src, dst) store indices."""
        out = []
        have = 1
        r = 0
        while have < self.n:
            step = 1 << r
            pairs = []
            for i in range(min(step, self.n)):
                j = i + step
                if j < self.n:
                    pairs.append(((self.root + i) % self.n, (self.root + j) % self.n))
            out.append(pairs)
            have = min(self.n, have * 2)
            r += 1
        return out

    def num_rounds(self) -> int:
        return math.ceil(math.log2(self.n)) if self.n > 1 else 0


def quantize_fp8_blockwise(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Weight [M, N] -> (fp8 e4m3 [M, N], fp32 scales [ceil(M/b), ceil(N/b)])."""
    M, N = w.shape
    mb, nb = math.ceil(M / block), math.ceil(N / block)
    pad = torch.zeros(mb * block, nb * block, dtype=torch.float32, device=w.device)
    pad[:M, :N] = w.float()
    tiles = pad.view(mb, block, nb, block)
    amax = tiles.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    fmax = torch.finfo(torch.float8_e4m3fn).max
    scale = amax / fmax
    q = (tiles / scale[:, None, :, None]).clamp(-fmax, fmax).to(torch.float8_e4m3fn)
    return q.view(mb * block, nb * block)[:M, :N].contiguous(), scale


def dequantize_fp8_blockwise(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    M, N = q.shape
    mb, nb = scale.shape
    pad = torch.zeros(mb * block, nb * block, dtype=torch.float32, device=q.device)
    pad[:M, :N] = q.float()
    t = pad.view(mb, block, nb, block) * scale[:, None, :, None]
    return t.view(mb * block, nb * block)[:M, :N]


def cast_train_to_gen(state: dict[str, torch.Tensor], gen_dtype: str = "bf16", block: int = 128) -> dict:
    """Generation-side copy of a state dict (2-D matrices quantised for fp8)."""
    if gen_dtype == "bf16":
        return {k: v.to(torch.bfloat16) for k, v in state.items()}
    if gen_dtype != "fp8":
        raise ValueError(f"unsupported gen dtype {gen_dtype}")
    out = {}
    for k, v in state.items():
        if v.dim() == 2 and min(v.shape) >= 16:
            q, s = quantize_fp8_blockwise(v, block)
            out[k] = q
            out[k + ".scale_inv"] = s
        else:
            out[k] = v.to(torch.bfloat16)
    return out
