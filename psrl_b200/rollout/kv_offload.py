"""KV-cache offload and cross-instance KV moves (C29 / N11 / K18).

``KVOffloadStore`` keeps evicted prefix blocks in pinned host memory, indexed by
the same content hashes the engine's prefix cache uses (so a later request
with that prefix can be served from host memory instead of recomputing it);
blocks can be pinned so they are never evicted.  ``transfer_direct`` copies a
request's blocks from one engine's cache into another's (a peer GPU over
NVLink via an IPC mapping, or the same GPU) — used when the router migrates a
partially generated request.  All moves are one ``kv_copy_blocks`` kernel over
every layer's K and V.  Reference: ``psrl/utils/kv_cache/manager.py``.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from .. import ops


def layer_ptrs(k_cache: list, v_cache: list, device) -> torch.Tensor:
    ptrs = [t.data_ptr() for t in k_cache] + [t.data_ptr() for t in v_cache]
    return torch.tensor(ptrs, dtype=torch.int64, device=device)


def block_bytes(k_cache: list) -> int:
    t = k_cache[0]
    return t[0].numel() * t.element_size()


def copy_blocks(src_k, src_v, dst_k, dst_v, src_blocks, dst_blocks, device=None) -> None:
    """dst[:, dst_blocks] <- src[:, src_blocks] for every layer's K and V."""
    if not src_blocks:
        return
    dev = device or dst_k[0].device
    if dev.type == "cuda":
        ops.ext().kv_copy_blocks(layer_ptrs(src_k, src_v, dev), layer_ptrs(dst_k, dst_v, dev),
                                 torch.tensor(src_blocks, dtype=torch.int32, device=dev),
                                 torch.tensor(dst_blocks, dtype=torch.int32, device=dev), block_bytes(src_k),
                                 src_k[0].shape[0], dst_k[0].shape[0])
        return
    for s, d in zip(list(src_k) + list(src_v), list(dst_k) + list(dst_v)):
        d[torch.tensor(dst_blocks)] = s[torch.tensor(src_blocks)].to(d.device)


class KVOffloadStore:
    def __init__(self, engine, capacity_blocks: int):
        self.engine = engine
        a = engine.args
        shape = (capacity_blocks, a.num_kv_heads, engine.block_size, a.head_dim)
        pin = engine.device.type == "cuda"
        self.k = [torch.zeros(shape, dtype=engine.dtype, pin_memory=pin) for _ in range(a.num_layers)]
        self.v = [torch.zeros(shape, dtype=engine.dtype, pin_memory=pin) for _ in range(a.num_layers)]
        self.capacity = capacity_blocks
        self.index: OrderedDict[int, int] = OrderedDict()      # content hash -> host slot
        self.free = list(range(capacity_blocks - 1, -1, -1))
        self.pinned: set[int] = set()

    def _slot(self) -> int | None:
        if self.free:
            return self.free.pop()
        for h in list(self.index):
            if h not in self.pinned:
                return self.index.pop(h)
        return None

    def offload(self, hashes: list[int], blocks: list[int]) -> int:
        """Copy device blocks (with their content hashes) to host; returns count."""
        src, dst, keep = [], [], []
        for h, b in zip(hashes, blocks):
            if h in self.index:
                self.index.move_to_end(h)
                continue
            s = self._slot()
            if s is None:
                break
            src.append(b)
            dst.append(s)
            keep.append(h)
        copy_blocks(self.engine.k_cache, self.engine.v_cache, self.k, self.v, src, dst, self.engine.device)
        for h, s in zip(keep, dst):
            self.index[h] = s
        return len(src)

    def onload(self, hashes: list[int], blocks: list[int]) -> int:
        """Copy the longest cached prefix of ``hashes`` into device ``blocks``."""
        src, dst = [], []
        for h, b in zip(hashes, blocks):
            s = self.index.get(h)
            if s is None:
                break
            src.append(s)
            dst.append(b)
        copy_blocks(self.k, self.v, self.engine.k_cache, self.engine.v_cache, src, dst, self.engine.device)
        return len(src)

    def pin(self, hashes) -> None:
        self.pinned |= set(hashes)

    def unpin(self, hashes) -> None:
        self.pinned -= set(hashes)

    def clear(self) -> None:
        self.index.clear()
        self.pinned.clear()
        self.free = list(range(self.capacity - 1, -1, -1))


def transfer_direct(src_engine, dst_engine, src_blocks: list[int], dst_blocks: list[int]) -> None:
    """Copy KV blocks between two engines (same or peer GPU)."""
    copy_blocks(src_engine.k_cache, src_engine.v_cache, dst_engine.k_cache, dst_engine.v_cache, src_blocks,
                dst_blocks, dst_engine.device)
