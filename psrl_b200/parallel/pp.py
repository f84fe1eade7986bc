"""Pipeline parallelism for the trainer: contiguous layer ranges per stage and a
1F1B micro-batch schedule over point-to-point sends (NCCL p2p on GPUs, gloo
on CPU).  The reference gets PP / VPP from Megatron's pipeline schedules
(``psrl/utils/config.py:119-126`` sizes the groups); pipeline send / recv stays
on NCCL p2p, overlapped with compute by the schedule.

Stage ``s`` of ``n`` owns decoder layers ``[s L / n, (s + 1) L / n)``; the first
stage also owns the embedding, the last the final norm and the LM head.  The
activations crossing a stage boundary are the residual stream pair
``(x, resid)`` of the packed micro-batch ([T, hidden] each); their gradients
come back the same way.  With tied embeddings the first and last stage both
hold the embedding matrix and :meth:`PipelineStage.reduce_tied_grads` adds
their two gradients (Megatron's embedding group).

Schedule per stage (``M`` micro-batches): ``n - s - 1`` warm-up forwards,
then one forward + one backward per step, then the remaining backwards; a
forward's send to the next stage and the matching backward's receive from it
are posted together (``batch_isend_irecv``) so neighbouring stages never wait
on each other's sends.  At most ``n - s`` micro-batches' activations are alive
on stage ``s``.

Virtual (interleaved) stages, ``virtual = v > 1``: the layers split into
``n v`` chunks and rank ``s`` holds chunks ``s, s + n, ..., s + (v - 1) n``, so
a micro-batch crosses every rank ``v`` times and the pipeline bubble shrinks by
``v`` (Megatron's interleaved schedule; the reference sizes it with
``virtual_pipeline_model_parallel_size``).  The per-rank order is the
interleaved 1F1B order of Narayanan et al. (SC'21): micro-batches in groups of
``n``, each group through chunks ``0 .. v-1`` forward and ``v-1 .. 0``
backward, ``2 (n - s - 1) + (v - 1) n`` warm-up forwards on rank ``s``.
:func:`interleaved_timetable` turns these orders into ticks by simulating all
ranks (every rank computes the same table): in each tick a rank runs its next
action if its input has arrived, and the activations / gradients made in the
tick are exchanged at its end in one ``batch_isend_irecv`` whose operations
every pair of ranks posts in the same order.  Nothing can deadlock or pair a
gradient with an activation, even when two ranks exchange both kinds.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops


def interleaved_timetable(n: int, v: int, M: int, forward_only: bool = False) -> list[tuple[list, list]]:
    """Ticks of the interleaved schedule for ``n`` ranks, ``v`` chunks per rank
    and ``M`` micro-batches.  Each tick is ``(actions, messages)``: actions[r]
    is ``None`` or ``(kind, mb, c)`` with kind ``"F"`` / ``"B"`` and ``c`` rank
    r's local chunk (global chunk ``c n + r``); messages are ``(src, dst, kind,
    mb, g)`` sent at the end of the tick, kind ``"act"`` (input of global chunk
    g) or ``"grad"`` (output gradient of global chunk g)."""
    nc = n * v
    groups = [list(range(g0, min(g0 + n, M))) for g0 in range(0, M, n)]
    fwd = [(mb, c) for grp in groups for c in range(v) for mb in grp]
    bwd = [(mb, c) for grp in groups for c in reversed(range(v)) for mb in grp]
    orders = []
    for r in range(n):
        if forward_only:
            orders.append([("F",) + x for x in fwd])
            continue
        w = min(len(fwd), 2 * (n - r - 1) + (v - 1) * n)
        seq = [("F",) + x for x in fwd[:w]]
        b = 0
        for f in range(w, len(fwd)):
            seq.append(("F",) + fwd[f])
            seq.append(("B",) + bwd[b])
            b += 1
        seq += [("B",) + x for x in bwd[b:]]
        orders.append(seq)
    ptr = [0] * n
    have: list[set] = [set() for _ in range(n)]     # messages delivered to each rank
    fdone: list[set] = [set() for _ in range(n)]
    ticks = []
    while any(ptr[r] < len(orders[r]) for r in range(n)):
        acts, msgs = [None] * n, []
        for r in range(n):
            if ptr[r] == len(orders[r]):
                continue
            kind, mb, c = orders[r][ptr[r]]
            g = c * n + r
            if kind == "F":
                ready = g == 0 or ("act", mb, g) in have[r]
            else:
                ready = (mb, c) in fdone[r] and (g == nc - 1 or ("grad", mb, g) in have[r])
            if not ready:
                continue
            acts[r] = (kind, mb, c)
            ptr[r] += 1
            if kind == "F":
                fdone[r].add((mb, c))
                if g < nc - 1:
                    msgs.append((r, (r + 1) % n, "act", mb, g + 1))
            elif g > 0:
                msgs.append((r, (r - 1) % n, "grad", mb, g - 1))
        if all(x is None for x in acts):
            raise RuntimeError("pipeline timetable made no progress (schedule bug)")
        for src, dst, kind, mb, g in msgs:
            have[dst].add((kind, mb, g))
        ticks.append((acts, msgs))
    return ticks


class PipelineStage:
    def __init__(self, model, group=None, virtual: int = 1):
        self.model = model
        self.group = group
        self.n = dist.get_world_size(group)
        self.s = dist.get_rank(group)
        self.ranks = [dist.get_global_rank(group, i) for i in range(self.n)] if group is not None else \
            list(range(self.n))
        a = model.args
        self.v = max(1, int(virtual))
        if self.v > 1 and self.n < 2:
            raise ValueError("virtual pipeline stages need at least two pipeline ranks")
        nc = self.n * self.v
        if a.num_layers < nc:
            raise ValueError(f"{a.num_layers} layers cannot fill {self.n} x {self.v} pipeline chunks")
        bounds = [round(i * a.num_layers / nc) for i in range(nc + 1)]
        # this rank's chunks: global chunk c n + s is local chunk c
        self.chunks = [(bounds[c * self.n + self.s], bounds[c * self.n + self.s + 1]) for c in range(self.v)]
        self.lo, self.hi = self.chunks[0]
        self.first, self.last = self.s == 0, self.s == self.n - 1
        # release what this stage does not run (names of the kept parameters are unchanged)
        for i in range(a.num_layers):
            if not any(lo <= i < hi for lo, hi in self.chunks):
                model.layers[i] = nn.Module()
        if not self.first and not (self.last and a.tie_word_embeddings):
            model.embed = None
        if not self.last:
            model.norm = None
            if hasattr(model, "lm_head"):
                model.lm_head = None
        self.dtype = next(p for p in model.parameters()).dtype
        self.device = next(p for p in model.parameters()).device
        # first + last stage group for the tied embedding (created on every rank: new_group is collective)
        self._tie_group = None
        if a.tie_word_embeddings and self.n > 1:
            self._tie_group = dist.new_group([self.ranks[0], self.ranks[-1]])

    def parameters(self):
        return [p for p in self.model.parameters()]

    # ------------------------------------------------------------------ p2p
    def _p2p(self, send_next=None, send_prev=None, recv_next=None, recv_prev=None):
        """Post the given sends / receives together and wait for them.
        recv_* are the number of rows T of a [T, hidden] (x, resid) pair."""
        h = self.model.args.hidden_size
        ops_, got_next, got_prev = [], None, None
        if recv_prev is not None:
            got_prev = [torch.empty(recv_prev, h, dtype=self.dtype, device=self.device) for _ in range(2)]
            ops_ += [dist.P2POp(dist.irecv, t, self.ranks[self.s - 1], self.group) for t in got_prev]
        if send_next is not None:
            ops_ += [dist.P2POp(dist.isend, t.contiguous(), self.ranks[self.s + 1], self.group) for t in send_next]
        if recv_next is not None:
            got_next = [torch.empty(recv_next, h, dtype=self.dtype, device=self.device) for _ in range(2)]
            ops_ += [dist.P2POp(dist.irecv, t, self.ranks[self.s + 1], self.group) for t in got_next]
        if send_prev is not None:
            ops_ += [dist.P2POp(dist.isend, t.contiguous(), self.ranks[self.s - 1], self.group) for t in send_prev]
        if ops_:
            for w in dist.batch_isend_irecv(ops_):
                w.wait()
        return got_next, got_prev

    # -------------------------------------------------------------- compute
    def _forward(self, mb, inputs, c: int = 0):
        """Run local chunk ``c`` of this stage on micro-batch ``mb``.  Returns
        (outputs, loss): outputs = (x, resid) unless this is the model's last
        chunk, which returns the loss."""
        m, a = self.model, self.model.args
        g = c * self.n + self.s
        if g == 0:
            x = m.embed(mb["ids"])
            if a.embed_scale:
                x = x * torch.tensor(a.embed_scale, dtype=x.dtype)
            resid = None
        else:
            x, resid = inputs
        lo, hi = self.chunks[c]
        for i in range(lo, hi):
            x, resid = m.layers[i](x, resid, mb["pos"], mb["cu"], mb["max"])
        if g != self.n * self.v - 1:
            return (x, resid), None
        h, _ = ops.rms_norm(x, m.norm, a.rms_eps, residual=resid)
        if a.value_head:
            return None, self.loss_fn(m.value(h).float().squeeze(-1), None, mb)
        lp, ent = ops.linear_logprob(h, m.lm_head_weight(), mb["labels"], mb.get("temperature", 1.0))
        return None, self.loss_fn(lp, ent, mb)

    def train_step(self, micro_batches: list[dict], loss_fn) -> list[float]:
        """Forward + backward of every micro-batch (gradients accumulate in
        ``.grad``).  Each micro-batch dict holds ``ids``, ``pos``, ``cu``,
        ``max`` and ``labels`` (the same on every stage); ``loss_fn(logprobs,
        entropy, mb)`` gives the scalar loss on the last stage.  Returns the
        last stage's losses (empty elsewhere)."""
        self.loss_fn = loss_fn
        if self.v > 1:
            return self._train_step_interleaved(micro_batches)
        M = len(micro_batches)
        warm = min(self.n - self.s - 1, M)
        saved: dict[int, tuple] = {}
        losses: list[float] = []
        T = [int(mb["ids"].shape[0]) for mb in micro_batches]

        def run_fwd(k, inputs):
            if inputs is not None:
                inputs = [t.requires_grad_(True) for t in inputs]
            out, loss = self._forward(micro_batches[k], inputs)
            saved[k] = (inputs, out, loss)
            if loss is not None:
                losses.append(float(loss.detach()))
            return out

        def run_bwd(k, grads):
            inputs, out, loss = saved.pop(k)
            if self.last:
                loss.backward()
            else:
                torch.autograd.backward([t for t in out], [g for g in grads])
            return [t.grad for t in inputs] if inputs is not None else None

        # warm-up forwards
        for k in range(warm):
            _, prev = self._p2p(recv_prev=None if self.first else T[k])
            out = run_fwd(k, prev)
            self._p2p(send_next=out)
        # steady state: forward k + warm, backward k
        for k in range(M - warm):
            f = k + warm
            _, prev = self._p2p(recv_prev=None if self.first else T[f])
            out = run_fwd(f, prev)
            if self.last:
                gin = run_bwd(k, None)
            else:
                nxt, _ = self._p2p(send_next=out, recv_next=T[k])
                gin = run_bwd(k, nxt)
            if not self.first:
                self._p2p(send_prev=gin)
        # cool-down backwards
        for k in range(M - warm, M):
            nxt, _ = self._p2p(recv_next=T[k])
            gin = run_bwd(k, nxt)
            if not self.first:
                self._p2p(send_prev=gin)
        return losses

    # ------------------------------------------------------- interleaved
    def _exchange(self, msgs, outbox: dict, inbox: dict, T: list[int]) -> None:
        """End-of-tick transfers: this rank's sends and receives among
        ``msgs``, posted in the table's order (the same on both ends)."""
        h = self.model.args.hidden_size
        ops_, got = [], []
        for src, dst, kind, mb, g in msgs:
            if src == self.s:
                for t in outbox.pop((kind, mb, g)):
                    ops_.append(dist.P2POp(dist.isend, t.contiguous(), self.ranks[dst], self.group))
            elif dst == self.s:
                bufs = [torch.empty(T[mb], h, dtype=self.dtype, device=self.device) for _ in range(2)]
                ops_ += [dist.P2POp(dist.irecv, t, self.ranks[src], self.group) for t in bufs]
                got.append(((kind, mb, g // self.n), bufs))
        if ops_:
            for w in dist.batch_isend_irecv(ops_):
                w.wait()
        for key, bufs in got:
            inbox[key] = bufs

    def _train_step_interleaved(self, micro_batches: list[dict]) -> list[float]:
        n, v, s = self.n, self.v, self.s
        M = len(micro_batches)
        T = [int(mb["ids"].shape[0]) for mb in micro_batches]
        saved: dict = {}
        inbox: dict = {}
        outbox: dict = {}
        losses: list[tuple[int, float]] = []
        for acts, msgs in interleaved_timetable(n, v, M):
            act = acts[s]
            if act is not None:
                kind, k, c = act
                g = c * n + s
                if kind == "F":
                    inputs = None if g == 0 else [t.requires_grad_(True) for t in inbox.pop(("act", k, c))]
                    out, loss = self._forward(micro_batches[k], inputs, c)
                    saved[(k, c)] = (inputs, out, loss)
                    if loss is not None:
                        losses.append((k, float(loss.detach())))
                    else:
                        outbox[("act", k, g + 1)] = list(out)
                else:
                    inputs, out, loss = saved.pop((k, c))
                    if loss is not None:
                        loss.backward()
                    else:
                        torch.autograd.backward(list(out), inbox.pop(("grad", k, c)))
                    if g > 0:
                        outbox[("grad", k, g - 1)] = [t.grad for t in inputs]
            self._exchange(msgs, outbox, inbox, T)
        return [x for _, x in sorted(losses)]

    @torch.no_grad()
    def _forward_only_interleaved(self, micro_batches: list[dict]) -> list[torch.Tensor]:
        n, s = self.n, self.s
        T = [int(mb["ids"].shape[0]) for mb in micro_batches]
        inbox: dict = {}
        outbox: dict = {}
        ys: dict = {}
        for acts, msgs in interleaved_timetable(n, self.v, len(micro_batches), forward_only=True):
            act = acts[s]
            if act is not None:
                _, k, c = act
                g = c * n + s
                out, y = self._forward(micro_batches[k], None if g == 0 else inbox.pop(("act", k, c)), c)
                if y is not None:
                    ys[k] = y
                else:
                    outbox[("act", k, g + 1)] = list(out)
            self._exchange(msgs, outbox, inbox, T)
        outs = []
        for k in range(len(micro_batches)):
            y = ys[k].float().contiguous() if self.last else torch.empty(T[k], dtype=torch.float32,
                                                                          device=self.device)
            dist.broadcast(y, self.ranks[-1], group=self.group)
            outs.append(y)
        return outs

    @torch.no_grad()
    def forward_only(self, micro_batches: list[dict]) -> list[torch.Tensor]:
        """Per-token outputs of every micro-batch (log-probs, or values for a
        value head), computed on the last stage and broadcast to every stage."""
        outs: list[torch.Tensor] = []
        self.loss_fn = lambda y, ent, mb: y
        if self.v > 1:
            return self._forward_only_interleaved(micro_batches)
        for mb in micro_batches:
            T = int(mb["ids"].shape[0])
            _, prev = self._p2p(recv_prev=None if self.first else T)
            out, y = self._forward(mb, prev)
            if not self.last:
                self._p2p(send_next=out)
                y = torch.empty(T, dtype=torch.float32, device=self.device)
            y = y.float().contiguous()
            dist.broadcast(y, self.ranks[-1], group=self.group)
            outs.append(y)
        return outs

    def broadcast_metrics(self, metrics: dict) -> dict:
        """The last stage's loss metrics on every stage (the other stages see no loss)."""
        box = [metrics]
        dist.broadcast_object_list(box, src=self.ranks[-1], group=self.group)
        out = dict(box[0])
        for k, v in metrics.items():
            if k not in out:
                out[k] = v
        return out

    def reduce_tied_grads(self, grad_of=None) -> None:
        """Tied embeddings: first and last stage add their gradients of the
        shared matrix (a two-rank all-reduce; every stage calls this).
        ``grad_of(param)`` returns the tensor holding a parameter's accumulated
        gradient when that is not ``param.grad`` (an optimizer's main-grad
        buffer)."""
        if self._tie_group is None:
            return
        if self.first or self.last:
            w = self.model.embed.weight
            g = grad_of(w) if grad_of is not None else None
            if g is None:
                if w.grad is None:
                    w.grad = torch.zeros_like(w)
                g = w.grad
            dist.all_reduce(g, group=self._tie_group)
