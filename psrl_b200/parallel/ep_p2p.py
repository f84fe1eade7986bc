"""Expert-parallel all-to-all over NVLink peer memory (K12), replacing NCCL's
``all_to_all_single`` on the dispatch and combine data path.

Every rank of the expert-parallel group owns two receive buffers (used in
turn) and a flag array, all mapped into every other rank (CUDA IPC).  One
all-to-all:

1. the send-count matrix M[src][dst] is known on every rank (an all-gather of
   P integers; the backward uses its transpose), so each rank knows where its
   rows go in every destination's buffer: after the rows of lower-ranked
   sources;
2. one kernel (``scatter_segments``) stores this rank's rows for destination d
   straight into d's receive buffer with 16-byte peer stores over NVLink;
3. a one-thread flag barrier (``peer_barrier``, bounded wait with an error
   status) makes every rank's stores visible;
4. the received rows are copied out of the buffer (autograd may keep them).

Ordering: a buffer is written again two calls later, after a barrier that each
reader reaches only once its stream has copied the rows out, so no write lands
in rows that are still being read.  Rows that would not fit the buffers go
through NCCL instead.  No TMA and no multicast: plain stores through the IPC
mappings.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import ops
from ..ops.gemm import _err


class PeerAllToAll:
    MAX_RANKS = 8

    def __init__(self, group, device, max_bytes: int, timeout_s: float = 2.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > self.MAX_RANKS:
            raise ValueError(f"the peer all-to-all covers up to {self.MAX_RANKS} ranks")
        self.device = torch.device(device)
        self.cap = int(max_bytes) // 16 * 16
        self.timeout_s = float(timeout_s)
        self.bufs = [torch.empty(self.cap, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.flags = torch.zeros(16 * self.MAX_RANKS, dtype=torch.int32, device=self.device)
        mine = {"bufs": [ops.ext().ipc_handle(b) for b in self.bufs], "flags": ops.ext().ipc_handle(self.flags),
                "device": self.device.index}
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self.peer_bufs = [[None] * self.world for _ in range(2)]
        peer_flags = []
        for r, h in enumerate(allh):
            if r == self.rank:
                for b in range(2):
                    self.peer_bufs[b][r] = self.bufs[b]
                peer_flags.append(self.flags)
                continue
            if int(h["device"]) != self.device.index:
                ops.ext().enable_peer_access(int(h["device"]))
            for b in range(2):
                hb, off = h["bufs"][b]
                self.peer_bufs[b][r] = ops.ext().ipc_open(hb, int(off), self.cap, torch.uint8, int(h["device"]))
            hf, off = h["flags"]
            peer_flags.append(ops.ext().ipc_open(hf, int(off), 16 * self.MAX_RANKS, torch.int32, int(h["device"])))
        slot = 16 * self.rank
        self.slot_in = [peer_flags[r][slot:slot + 1] for r in range(self.world)]
        self.own = [self.flags[16 * r:16 * r + 1] for r in range(self.world)]
        self.epoch = 0
        self.calls = 0
        self.stats = {"calls": 0, "bytes": 0, "nccl_fallbacks": 0}

    def counts(self, send: list[int]) -> list[list[int]]:
        """Send-count matrix M[src][dst] from every rank's send counts."""
        t = torch.tensor(send, dtype=torch.int64, device=self.device)
        out = torch.empty(self.world * self.world, dtype=torch.int64, device=self.device)
        dist.all_gather_into_tensor(out, t, group=self.group)
        m = out.view(self.world, self.world).tolist()
        return m

    def __call__(self, x: torch.Tensor, M: list[list[int]]) -> torch.Tensor:
        """Rows of ``x`` grouped by destination (this rank sends M[rank][d] to
        d) -> the rows every source sends here, grouped by source."""
        P, me = self.world, self.rank
        rest = tuple(x.shape[1:])
        row = math.prod(rest) * x.element_size()
        recv = [M[s][me] for s in range(P)]
        n_out = sum(recv)
        fits = row % 16 == 0 and all(sum(M[s][d] for s in range(P)) * row <= self.cap for d in range(P))
        if not fits:
            self.stats["nccl_fallbacks"] += 1
            out = x.new_empty((n_out,) + rest)
            dist.all_to_all_single(out, x.contiguous(), recv, list(M[me]), group=self.group)
            return out
        buf = self.calls & 1
        self.calls += 1
        xs = x.contiguous().view(torch.uint8).reshape(-1) if x.numel() else x.new_empty(0).view(torch.uint8)
        dsts, soffs, lens = [], [], []
        src_row = 0
        for d in range(P):
            n = M[me][d]
            if n:
                dst_row = sum(M[s][d] for s in range(me))
                dsts.append(self.peer_bufs[buf][d][dst_row * row:(dst_row + n) * row])
                soffs.append(src_row * row)
                lens.append(n * row)
            src_row += n
        if dsts:
            ops.ext().scatter_segments(xs, dsts, soffs, lens)
        self.epoch += 1
        ops.ext().peer_barrier(self.slot_in, self.own, self.epoch, self.timeout_s, _err(self.device))
        self.stats["calls"] += 1
        self.stats["bytes"] += sum(lens)
        return self.bufs[buf][: n_out * row].view(x.dtype).view((n_out,) + rest).clone()


class _PeerA2AFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, M, a2a):
        ctx.M, ctx.a2a = M, a2a
        return a2a(x, M)

    @staticmethod
    def backward(ctx, g):
        Mt = [list(col) for col in zip(*ctx.M)]          # every row goes back to its sender
        return ctx.a2a(g.contiguous(), Mt), None, None


def peer_all_to_all(x: torch.Tensor, M: list[list[int]], a2a: PeerAllToAll) -> torch.Tensor:
    return _PeerA2AFn.apply(x, M, a2a)
