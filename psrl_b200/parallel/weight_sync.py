"""Trainer → rollout weight synchronisation through the Parameter Server store (K17, N6).

The reference moves weights train GPU → pinned-CPU PS (NIXL write) → rollout
GPU (NIXL read) with a meta-server comm plan (``psrl/utils/nixl/*``).  Here:

* **Store** — every trainer rank keeps a *published* copy of the full
  parameters in its own HBM (``ps_mode=hbm``; a shared-memory host tensor for
  ``ps_mode=cpu``).  The trainer writes it under the PS exclusive-push lock
  right after the optimizer step; training never waits for readers.
* **Layout** — the store uses the trainer's flat layout
  (:attr:`FlatShardedDP.layout`), which is already the fused rollout layout
  (qkv / gate_up stacked), so at TP=1 the rollout weights are views into one
  flat buffer of the same layout and the "transform" is the identity.
* **Pull** — a rollout rank maps every trainer's store once (CUDA IPC) and
  pulls disjoint slices from different trainers in ONE kernel
  (``copy_segments``: 16-byte peer loads over NVLink straight into the engine's
  weights; no copy engine, no staging buffer, no TMA multicast), under the PS
  shared-pull lock.  Spreading the slices over all trainers keeps every
  trainer's NVLink egress busy.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops


@dataclass
class WeightLayout:
    entries: list            # (name, shape, offset) in elements
    total: int
    dtype: torch.dtype

    @classmethod
    def from_dp(cls, dp) -> "WeightLayout":
        return cls(list(dp.layout), int(dp.total), dp.flat.dtype)

    def views(self, flat: torch.Tensor) -> dict[str, torch.Tensor]:
        out = {}
        for name, shape, off in self.entries:
            n = 1
            for s in shape:
                n *= s
            out[name] = flat[off: off + n].view(shape)
        return out

    @property
    def nbytes(self) -> int:
        return self.total * torch.finfo(self.dtype).bits // 8


class WeightStore:
    """Trainer-side published copy of the parameters."""

    def __init__(self, layout: WeightLayout, device, mode: str = "hbm"):
        self.layout = layout
        self.mode = mode
        self.device = torch.device(device)
        if mode == "hbm":
            if self.device.type != "cuda":
                raise ValueError("ps_mode=hbm needs a CUDA device")
            self.flat = torch.empty(layout.total, dtype=layout.dtype, device=self.device)
        else:
            self.flat = torch.empty(layout.total, dtype=layout.dtype).share_memory_()
        self.version = -1

    @torch.no_grad()
    def publish(self, src_flat: torch.Tensor, version: int) -> None:
        if self.mode == "hbm":
            nbytes = self.layout.nbytes
            ops.ext().copy_segments(self.flat, [src_flat], [0], [0], [nbytes])
        else:
            self.flat.copy_(src_flat.to("cpu", non_blocking=False))
        self.version = int(version)

    def descriptor(self) -> dict:
        if self.mode == "hbm":
            handle, off = ops.ext().ipc_handle(self.flat)
            return {"kind": "ipc", "handle": handle, "offset": off, "numel": self.layout.total,
                    "dtype": str(self.layout.dtype).replace("torch.", ""), "device": self.device.index}
        return {"kind": "shm", "tensor": self.flat}


def open_store(desc: dict) -> torch.Tensor:
    """Map a trainer's store in this process (a view of peer HBM or shared memory)."""
    if desc["kind"] == "ipc":
        dt = getattr(torch, desc["dtype"])
        return ops.ext().ipc_open(desc["handle"], int(desc["offset"]), int(desc["numel"]), dt, int(desc["device"]))
    return desc["tensor"]


class WeightPuller:
    """Rollout-side: pulls the store slices from all trainers into ``dst_flat``."""

    def __init__(self, layout: WeightLayout, descriptors: list[dict], dst_flat: torch.Tensor):
        self.layout = layout
        self.dst = dst_flat
        self.srcs = [open_store(d) for d in descriptors]
        self.gpu = dst_flat.is_cuda
        if self.gpu:
            me = dst_flat.device.index
            for d in descriptors:
                if d["kind"] == "ipc" and int(d["device"]) != me:
                    ops.ext().enable_peer_access(int(d["device"]))
        T = len(self.srcs)
        esz = torch.finfo(layout.dtype).bits // 8
        total_b = layout.total * esz
        # split into T slices aligned to 16 bytes
        step = (total_b // T) // 16 * 16
        self.plan = []
        for j in range(T):
            lo = j * step
            hi = total_b if j == T - 1 else (j + 1) * step
            self.plan.append((j, lo, hi - lo))

    @torch.no_grad()
    def pull(self) -> int:
        if self.gpu:
            ops.ext().copy_segments(self.dst, [self.srcs[j] for j, _, _ in self.plan],
                                    [lo for _, lo, _ in self.plan], [lo for _, lo, _ in self.plan],
                                    [n for _, _, n in self.plan])
        else:
            esz = self.dst.element_size()
            for j, lo, n in self.plan:
                a, b = lo // esz, (lo + n) // esz
                self.dst[a:b].copy_(self.srcs[j][a:b])
        return self.layout.nbytes


class ShardedWeightPuller:
    """Rollout-side pull from trainers whose stores hold different parameter
    sets (pipeline stages: each stage publishes only its layers).  Every
    tensor of the engine's full layout is copied from a store that holds it
    (round-robin over the data-parallel replicas of its stage, so the load
    spreads over their NVLink links), straight into its place in the engine's
    flat buffer: the store layout is transformed into the engine layout by the
    copy itself, with no assembly on the trainers.  Runs of tensors that are
    contiguous on both sides merge into one segment; the segments go through
    ``copy_segments`` 16 per launch."""

    MAX_SEG = 16

    def __init__(self, layout: WeightLayout, descriptors: list[dict], dst_flat: torch.Tensor):
        self.layout = layout
        self.dst = dst_flat
        self.srcs = [open_store(d) for d in descriptors]
        self.gpu = dst_flat.is_cuda
        if self.gpu:
            me = dst_flat.device.index
            for d in descriptors:
                if d["kind"] == "ipc" and int(d["device"]) != me:
                    ops.ext().enable_peer_access(int(d["device"]))
        esz = torch.finfo(layout.dtype).bits // 8
        owners: dict[str, list] = {}
        for j, d in enumerate(descriptors):
            for name, shape, off in d["entries"]:
                owners.setdefault(name, []).append((j, int(off)))
        segs, turn = [], {}
        for name, shape, off in layout.entries:
            if name not in owners:
                raise KeyError(f"no trainer store holds {name}")
            cands = owners[name]
            k = turn.get(len(cands), 0)
            turn[len(cands)] = k + 1
            j, src = cands[k % len(cands)]
            n = 1
            for s in shape:
                n *= s
            seg = [j, src * esz, int(off) * esz, n * esz]
            last = segs[-1] if segs else None
            if last and last[0] == j and last[1] + last[3] == seg[1] and last[2] + last[3] == seg[2]:
                last[3] += seg[3]
            else:
                segs.append(seg)
        self.segments = [tuple(s) for s in segs]       # (store, src byte, dst byte, bytes)

    @torch.no_grad()
    def pull(self) -> int:
        if self.gpu:
            for i in range(0, len(self.segments), self.MAX_SEG):
                part = self.segments[i:i + self.MAX_SEG]
                ops.ext().copy_segments(self.dst, [self.srcs[j] for j, _, _, _ in part], [d for _, _, d, _ in part],
                                        [s for _, s, _, _ in part], [n for _, _, _, n in part])
        else:
            esz = self.dst.element_size()
            for j, s, d, n in self.segments:
                self.dst[d // esz:(d + n) // esz].copy_(self.srcs[j][s // esz:(s + n) // esz])
        return sum(n for _, _, _, n in self.segments)
