"""Paged KV-cache block manager with prefix caching.

* The device cache is one tensor per layer and per K/V of shape
  ``[num_blocks, nkv, block_size, head_dim]`` (a (block, head) pair is one
  contiguous ``block_size x head_dim`` tile, which is what the decode and
  prefill kernels load).
* Full blocks are content-addressed by a hash chain over (parent hash, the
  block's tokens, weight version); a new request whose prompt starts with a
  cached chain reuses those blocks (multi-turn prefix reuse, K1/K2).
* Blocks are reference counted; blocks whose count drops to zero stay in the
  content index and are reclaimed in LRU order when the free list is empty.
* The weight version is part of the hash, so a weight update never serves KV
  computed by older weights.
"""

from __future__ import annotations

from collections import OrderedDict

import torch


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        self.ref = [0] * self.num_blocks
        self.free: list[int] = list(range(self.num_blocks - 1, -1, -1))
        self.hash_of: dict[int, int] = {}           # block -> content hash (full cached blocks)
        self.block_of: dict[int, int] = {}          # content hash -> block
        self.evictable: OrderedDict[int, None] = OrderedDict()  # ref==0 cached blocks in LRU order
        self.version = 0
        self.hits = 0
        self.queries = 0

    # ------------------------------------------------------------ capacity
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def usage(self) -> float:
        return 1.0 - self.num_free() / max(1, self.num_blocks)

    def _take(self) -> int:
        if self.free:
            b = self.free.pop()
        elif self.evictable:
            b, _ = self.evictable.popitem(last=False)
            h = self.hash_of.pop(b)
            self.block_of.pop(h, None)
        else:
            raise MemoryError("KV cache out of blocks")
        self.ref[b] = 1
        return b

    def _release(self, b: int) -> None:
        self.ref[b] -= 1
        if self.ref[b] > 0:
            return
        if b in self.hash_of:
            self.evictable[b] = None
        else:
            self.free.append(b)

    # --------------------------------------------------------------- hashing
    def chain_hashes(self, tokens: list[int]) -> list[int]:
        hs, parent = [], hash(("v", self.version))
        bs = self.block_size
        for i in range(len(tokens) // bs):
            parent = hash((parent, tuple(tokens[i * bs: (i + 1) * bs])))
            hs.append(parent)
        return hs

    def set_version(self, version: int) -> None:
        """New weights: drop the content index (cached KV is stale)."""
        self.version = int(version)
        for b in list(self.evictable):
            self.free.append(b)
        self.evictable.clear()
        self.hash_of.clear()
        self.block_of.clear()

    # --------------------------------------------------------- allocation
    def match_prefix(self, tokens: list[int]) -> list[int]:
        """Cached blocks covering a prefix of ``tokens`` (refs taken)."""
        self.queries += 1
        out = []
        for h in self.chain_hashes(tokens):
            b = self.block_of.get(h)
            if b is None:
                break
            if self.ref[b] == 0:
                self.evictable.pop(b, None)
            self.ref[b] += 1
            out.append(b)
        if out:
            self.hits += 1
        return out

    def allocate(self, n: int) -> list[int]:
        if n > self.num_free():
            raise MemoryError("KV cache out of blocks")
        return [self._take() for _ in range(n)]

    def can_allocate(self, n: int) -> bool:
        return n <= self.num_free()

    def release(self, blocks: list[int]) -> None:
        for b in blocks:
            self._release(b)

    def register_full_blocks(self, blocks: list[int], tokens: list[int], start_block: int = 0) -> None:
        """Publish the content hashes of full blocks so later requests can reuse them."""
        hs = self.chain_hashes(tokens)
        for i in range(start_block, min(len(hs), len(blocks))):
            b, h = blocks[i], hs[i]
            if b in self.hash_of or h in self.block_of:
                continue
            self.hash_of[b] = h
            self.block_of[h] = b


def allocate_kv_tensors(num_layers: int, num_blocks: int, nkv: int, block_size: int, head_dim: int, dtype, device,
                        pool=None, tag: str = "kv"):
    """Two lists (K, V) of per-layer [num_blocks, nkv, block_size, head_dim] tensors.
    With ``pool`` (:class:`psrl_b200.parallel.memory.MemoryPool`) the cache lives
    in one driver virtual-memory region per tensor under ``tag``, so the engine
    can release its physical memory while asleep and keep the addresses."""
    shape = (num_blocks, nkv, block_size, head_dim)
    if pool is not None:
        k = [pool.tensor(tag, shape, dtype) for _ in range(num_layers)]
        v = [pool.tensor(tag, shape, dtype) for _ in range(num_layers)]
        for t in k + v:
            t.zero_()
        return k, v
    k = [torch.zeros(*shape, dtype=dtype, device=device) for _ in range(num_layers)]
    v = [torch.zeros(*shape, dtype=dtype, device=device) for _ in range(num_layers)]
    return k, v
