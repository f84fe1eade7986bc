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

    @torch.no_grad()
    def publish_parts(self, parts: list[torch.Tensor], version: int) -> None:
        """Publish several flat buffers back to back (a tensor-parallel rank's
        replicated and sharded parameters)."""
        esz = torch.finfo(self.layout.dtype).bits // 8
        offs, o = [], 0
        for t in parts:
            offs.append(o)
            o += t.numel() * esz
        if self.mode == "hbm":
            ops.ext().copy_segments(self.flat, list(parts), offs, [0] * len(parts), [t.numel() * esz for t in parts])
        else:
            for t, off in zip(parts, offs):
                self.flat[off // esz: off // esz + t.numel()].copy_(t.to("cpu"))
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
    sets, writing the engine's full layout directly (no assembly on the
    trainers):

    * pipeline stages: a store holds whole tensors of its layers (descriptor
      ``entries`` with the full names and shapes); each tensor is read from a
      store that holds it, round-robin over the stage's data-parallel replicas;
    * tensor-parallel ranks: a store holds this rank's shards (``entries`` with
      the local names and shapes plus ``tp_rank`` / ``tp_world``); every
      sharded tensor is assembled from all TP ranks' shards as it is copied:
      column-parallel row ranges (q | k | v heads, gate | up halves) are
      contiguous blocks, row-parallel column ranges (O, down) are 2-D blocks
      with their own row strides (``models.converters.tp_slices`` gives the
      pieces).  Replicated tensors come from any rank.  Among the stores that
    hold a piece, the comm plan's rule picks the sender (``comm_plan.least_loaded``:
    best link, then fewest bytes so far).

    On CUDA the whole plan runs as ONE kernel (``copy_rows``: a device table of
    2-D byte blocks, 16-byte loads from the trainers' HBM over NVLink)."""

    def __init__(self, layout: WeightLayout, descriptors: list[dict], dst_flat: torch.Tensor, args=None):
        from .assemble import engine_name
        from ..models.converters import tp_slices
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
        whole: dict[str, list] = {}        # engine name -> [(store, offset)]
        shards: dict[str, dict] = {}       # engine name -> {tp rank: [(store, offset, local shape)]}
        full_shape = {n: tuple(sh) for n, sh, _ in layout.entries}
        for j, d in enumerate(descriptors):
            tp = d.get("tp_world", 1)
            for name, shape, off in d["entries"]:
                en = engine_name(name)
                # a TP shard: renamed (dense TP modules) or narrower than the full
                # tensor under the same name (tensor-parallel experts)
                if tp > 1 and (en != name or tuple(shape) != full_shape.get(en, tuple(shape))):
                    shards.setdefault(en, {}).setdefault(int(d["tp_rank"]), []).append((j, int(off), tuple(shape)))
                else:
                    whole.setdefault(en, []).append((j, int(off)))
        from .comm_plan import least_loaded
        blocks = []
        load: dict[int, int] = {}          # bytes assigned to each store so far
        link = {j: ("self" if d.get("device") == (dst_flat.device.index if self.gpu else None) else "nvlink")
                for j, d in enumerate(descriptors)}

        def pick(cands, nbytes):
            # the comm plan's rule: best link, then the least-loaded holder, so the
            # egress of every trainer GPU holding a tensor is used evenly
            j = least_loaded([c[0] for c in cands], load, link)
            load[j] = load.get(j, 0) + nbytes
            return next(c for c in cands if c[0] == j)

        for name, shape, off in layout.entries:
            n = 1
            for x in shape:
                n *= x
            dst0 = int(off) * esz
            if name in shards:
                per = shards[name]
                P = len(per)
                full = tuple(shape)
                for r in range(P):
                    j, loff, lshape = pick(per[r], n * esz // P)
                    acc = 0
                    for dim, start, length in tp_slices(name, full, args, r, P):
                        # the piece is `outer` rows (one per index of the leading
                        # dimensions) of length x inner contiguous elements
                        inner = 1
                        for x in full[dim + 1:]:
                            inner *= x
                        outer = 1
                        for x in full[:dim]:
                            outer *= x
                        src, dst = (loff + acc * inner) * esz, dst0 + start * inner * esz
                        if outer == 1:
                            blocks.append((j, src, dst, 1, length * inner * esz, 0, 0))
                        else:
                            blocks.append((j, src, dst, outer, length * inner * esz, lshape[dim] * inner * esz,
                                           full[dim] * inner * esz))
                        acc += length
            elif name in whole:
                j, soff = pick(whole[name], n * esz)
                blocks.append((j, soff * esz, dst0, 1, n * esz, 0, 0))
            else:
                raise KeyError(f"no trainer store holds {name}")
        self._set_blocks(blocks)

    def _set_blocks(self, blocks: list) -> None:
        """Merge contiguous one-row blocks, check alignment and build the
        device table of the copy kernel."""
        # merge contiguous one-row blocks (same store, adjacent on both sides)
        merged = []
        for b in blocks:
            last = merged[-1] if merged else None
            if last and b[3] == 1 and last[3] == 1 and last[0] == b[0] and last[1] + last[4] == b[1] \
                    and last[2] + last[4] == b[2]:
                merged[-1] = (last[0], last[1], last[2], 1, last[4] + b[4], 0, 0)
            else:
                merged.append(b)
        for b in merged:
            if b[4] % 16 or b[1] % 16 or b[2] % 16 or (b[3] > 1 and (b[5] % 16 or b[6] % 16)):
                raise ValueError(f"weight pull block {b} is not 16-byte aligned")
        self.blocks = merged          # (store, src byte, dst byte, rows, row bytes, src stride, dst stride)
        if self.gpu:
            tab = torch.tensor([[int(self.srcs[j].data_ptr()) + s, d, rows, rb // 16, ss, ds]
                                for j, s, d, rows, rb, ss, ds in merged], dtype=torch.int64)
            start = torch.zeros(len(merged) + 1, dtype=torch.int64)
            start[1:] = torch.tensor([rows * (rb // 16) for _, _, _, rows, rb, _, _ in merged],
                                     dtype=torch.int64).cumsum(0)
            self.table = tab.to(self.dst.device)
            self.start = start.to(self.dst.device)

    @torch.no_grad()
    def pull(self) -> int:
        if self.gpu:
            ops.ext().copy_rows(self.dst, self.table, self.start)
        else:
            dst = self.dst.view(torch.uint8)
            for j, s, d, rows, rb, ss, ds in self.blocks:
                src = self.srcs[j].view(torch.uint8)
                if rows == 1:
                    dst[d:d + rb].copy_(src[s:s + rb])
                else:
                    dst.as_strided((rows, rb), (ds, 1), d).copy_(src.as_strided((rows, rb), (ss, 1), s))
        return sum(rows * rb for _, _, _, rows, rb, _, _ in self.blocks)


class EngineShardPuller(ShardedWeightPuller):
    """A tensor-parallel rollout rank's pull from whole-tensor trainer stores
    (data-parallel trainers), or from the stores of a dense tensor-parallel
    trainer of the same TP size (whole shards of the same rank): only this
    rank's slices of every tensor
    (``parallel.tp.engine_slices``: heads, MLP width, whole experts, the KV head
    it reads when there are more ranks than KV heads; replicated tensors whole)
    are copied, straight into the engine's shard tensors, in one kernel on
    CUDA.  ``tensors`` maps each name to its view of the shard flat buffer."""

    def __init__(self, layout: WeightLayout, descriptors: list[dict], args, tp_rank: int, tp_world: int,
                 device=None):
        from ..parallel.tp import engine_slices
        from .comm_plan import least_loaded
        esz = torch.finfo(layout.dtype).bits // 8
        pieces, local, total = {}, {}, 0
        for name, shape, _ in layout.entries:
            sl = engine_slices(name, tuple(shape), args, tp_rank, tp_world)
            lshape = list(shape)
            lshape[sl[0][0]] = sum(x[2] for x in sl)
            pieces[name], local[name] = sl, (tuple(lshape), total)
            n = 1
            for x in lshape:
                n *= x
            total += -(-n * esz // 16) * 16 // esz          # every shard starts on 16 bytes
        self.layout = layout
        self.srcs = [open_store(d) for d in descriptors]
        self.dst = torch.empty(total, dtype=layout.dtype,
                               device=device if device is not None else self._device_for(descriptors))
        self.gpu = self.dst.is_cuda
        if self.gpu:
            me = self.dst.device.index
            for d in descriptors:
                if d["kind"] == "ipc" and int(d["device"]) != me:
                    ops.ext().enable_peer_access(int(d["device"]))
        self.tensors = {}
        for name, (lshape, off) in local.items():
            n = 1
            for x in lshape:
                n *= x
            self.tensors[name] = self.dst[off:off + n].view(lshape)
        link = {j: ("self" if d.get("device") == (self.dst.device.index if self.gpu else None) else "nvlink")
                for j, d in enumerate(descriptors)}
        load: dict[int, int] = {}
        blocks = []
        if any("entries" in d for d in descriptors):
            # tensor-parallel trainer stores of the same TP size (dense model):
            # engine rank r's shard of every tensor is trainer rank r's, copied whole;
            # replicated tensors come from the least-loaded store
            from .assemble import engine_name
            held: dict[str, list] = {}
            for j, d in enumerate(descriptors):
                for nm, shp, o in d["entries"]:
                    held.setdefault(engine_name(nm), []).append((j, int(d.get("tp_rank", 0)), tuple(shp), int(o)))
            for name, shape, _ in layout.entries:
                lshape, loff = local[name]
                n = 1
                for x in lshape:
                    n *= x
                cands = [c for c in held.get(name, []) if c[2] == lshape and (c[2] == tuple(shape) or c[1] == tp_rank)]
                if not cands:
                    raise KeyError(f"no trainer store holds rank {tp_rank}'s {name} {lshape}")
                j = least_loaded([c[0] for c in cands], load, link)
                load[j] = load.get(j, 0) + n * esz
                o = next(c[3] for c in cands if c[0] == j)
                blocks.append((j, o * esz, loff * esz, 1, n * esz, 0, 0))
            self._set_blocks(blocks)
            return
        for name, shape, off in layout.entries:
            full = tuple(shape)
            lshape, loff = local[name]
            acc = 0
            for dim, start, length in pieces[name]:
                inner = 1
                for x in full[dim + 1:]:
                    inner *= x
                outer = 1
                for x in full[:dim]:
                    outer *= x
                nbytes = outer * length * inner * esz
                j = least_loaded(list(range(len(descriptors))), load, link)
                load[j] = load.get(j, 0) + nbytes
                src, dst = (int(off) + start * inner) * esz, (loff + acc * inner) * esz
                if outer == 1:
                    blocks.append((j, src, dst, 1, length * inner * esz, 0, 0))
                else:
                    blocks.append((j, src, dst, outer, length * inner * esz, full[dim] * inner * esz,
                                   lshape[dim] * inner * esz))
                acc += length
        self._set_blocks(blocks)

    @staticmethod
    def _device_for(descriptors):
        if torch.cuda.is_available() and any(d.get("kind") == "ipc" for d in descriptors):
            return torch.device("cuda", torch.cuda.current_device())
        return torch.device("cpu")
