"""Weight-transfer planning between differently sharded layouts (C17).

Every participant describes how it shards each tensor (a ``Sharding``: the
tensor is split along one dim into ``n`` equal parts, this participant owns
part ``index``; replicated tensors use ``n = 1``).  Planning:

1. **finest shard mesh** — for a tensor sharded ``a`` ways by the senders and
   ``b`` ways by a receiver, the unit of transfer is ``lcm(a, b)`` pieces
   along the shard dim, so every piece has exactly one sender part and one
   receiver part;
2. **candidate senders** — a piece can come from any sender replica holding it;
3. **load balancing** — pieces are assigned greedily to the candidate with the
   lowest accumulated bytes, preferring higher-priority links
   (NVLink > PCIe > network), which spreads the egress over all trainer GPUs;
4. **contiguous merging** — pieces from the same sender that are adjacent in
   both source and destination memory are merged into one segment, so the pull
   kernel gets few, large segments.

Reference: ``psrl/utils/nixl/{nixl_spec,comm_plan,network_topology}.py``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

LINK_PRIORITY = {"self": 0, "nvlink": 1, "pcie": 2, "ib": 3, "tcp": 4}


@dataclass(frozen=True)
class Sharding:
    dim: int = 0
    n: int = 1
    index: int = 0


@dataclass
class TensorSpec:
    name: str
    shape: tuple
    itemsize: int = 2


@dataclass
class Segment:
    tensor: str
    src: int                 # sender id
    src_off: int             # byte offset inside the sender's local shard of the tensor
    dst_off: int             # byte offset inside the receiver's local shard
    nbytes: int


@dataclass
class CommPlan:
    segments: list = field(default_factory=list)

    def bytes_per_sender(self) -> dict:
        out: dict = {}
        for s in self.segments:
            out[s.src] = out.get(s.src, 0) + s.nbytes
        return out

    def total_bytes(self) -> int:
        return sum(s.nbytes for s in self.segments)


def _row_bytes(shape: tuple, dim: int, itemsize: int) -> int:
    """Bytes of one index step along ``dim`` when ``dim`` is the outermost split
    (only dim 0 splits are contiguous; others are handled per outer row)."""
    inner = 1
    for s in shape[dim + 1:]:
        inner *= s
    return inner * itemsize


def least_loaded(cands: list[int], load: dict, link: dict | None = None) -> int:
    """Sender for the next piece: the best link class first (NVLink before PCIe
    before the network), then the fewest bytes assigned so far."""
    link = link or {}
    return min(cands, key=lambda c: (LINK_PRIORITY.get(link.get(c, "nvlink"), 9), load.get(c, 0), c))


def plan_transfer(specs: list[TensorSpec], senders: dict[int, dict[str, Sharding]],
                  receiver: dict[str, Sharding], link: dict[int, str] | None = None) -> CommPlan:
    """Plan the segments one receiver must pull.

    ``senders[sid][name]`` is sender ``sid``'s sharding of tensor ``name``;
    ``receiver[name]`` the receiver's.  Offsets are in each side's *local*
    shard (a contiguous buffer holding only its part).
    """
    link = link or {}
    load: dict[int, int] = {sid: 0 for sid in senders}
    plan = CommPlan()
    for spec in specs:
        r = receiver[spec.name]
        holders = [(sid, sh[spec.name]) for sid, sh in senders.items() if spec.name in sh]
        if not holders:
            raise KeyError(f"no sender holds {spec.name}")
        dims = {h.dim for _, h in holders if h.n > 1} | ({r.dim} if r.n > 1 else set())
        if len(dims) > 1:
            raise ValueError(f"{spec.name}: mixed shard dims {dims} are not supported")
        dim = dims.pop() if dims else 0
        if dim != 0 and any(h.n > 1 for _, h in holders) and r.n > 1:
            raise ValueError(f"{spec.name}: both sides sharded along non-leading dim {dim}")
        a = max(h.n for _, h in holders)
        L = math.lcm(a, r.n)
        extent = spec.shape[dim]
        if extent % L:
            raise ValueError(f"{spec.name}: dim {dim} ({extent}) not divisible by {L}")
        piece = extent // L
        outer = 1
        for s in spec.shape[:dim]:
            outer *= s
        rowb = _row_bytes(spec.shape, dim, spec.itemsize)
        for p in range(L):
            if p * r.n // L != r.index:
                continue                       # piece not owned by this receiver
            cands = [(sid, h) for sid, h in holders if h.n == 1 or p * h.n // L == h.index]
            sid = least_loaded([c[0] for c in cands], load, link)
            h = dict(cands)[sid]
            # piece p covers rows [p*piece, (p+1)*piece) along dim
            src_first = p * piece - (h.index * (extent // h.n) if h.n > 1 else 0)
            dst_first = p * piece - r.index * (extent // r.n)
            src_extent = extent // h.n if h.n > 1 else extent
            dst_extent = extent // r.n
            for o in range(outer):
                nb = piece * rowb
                plan.segments.append(Segment(spec.name, sid, (o * src_extent + src_first) * rowb,
                                             (o * dst_extent + dst_first) * rowb, nb))
                load[sid] += nb
    plan.segments = merge_contiguous(plan.segments)
    return plan


def merge_contiguous(segs: list[Segment]) -> list[Segment]:
    out: list[Segment] = []
    for s in sorted(segs, key=lambda x: (x.tensor, x.src, x.src_off)):
        if out:
            t = out[-1]
            if t.tensor == s.tensor and t.src == s.src and t.src_off + t.nbytes == s.src_off and \
                    t.dst_off + t.nbytes == s.dst_off:
                t.nbytes += s.nbytes
                continue
        out.append(Segment(s.tensor, s.src, s.src_off, s.dst_off, s.nbytes))
    return out


@dataclass
class NetworkTopology:
    """Link type between participants (defaults: same node = NVLink)."""
    node_of: dict = field(default_factory=dict)
    nvlink_gbs: float = 900.0
    pcie_gbs: float = 128.0
    ib_gbps: float = 200.0

    def link(self, a: int, b: int) -> str:
        if a == b:
            return "self"
        return "nvlink" if self.node_of.get(a, 0) == self.node_of.get(b, 0) else "ib"

    def bandwidth_gbs(self, kind: str) -> float:
        return {"self": 3000.0, "nvlink": self.nvlink_gbs, "pcie": self.pcie_gbs, "ib": self.ib_gbps / 8}.get(kind, 1.0)
