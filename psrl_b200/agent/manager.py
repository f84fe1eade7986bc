"""Agent-loop manager: the driver-side dispatcher of the asynchronous pipeline (C12).

Responsibilities (reference ``psrl/workers/agent_loop/manager.py``):

1. **Dispatch-ahead bound** — prompt groups are released in order only while
   ``expected_ps_version <= ps_version`` with
   ``expected = initial + max(dispatched - min(eta, max_ahead) * buffer_size, 0) // buffer_size``
   (``_get_expected_ps_version`` :636-652), so rollout never runs more than
   ``min(eta, max_dispatch_ahead)`` buffers ahead of training.
2. **Admission (Reserve)** — a rollout instance asks for work with its weight
   version; each request is reserved in the PS at that version before it is
   handed out (the role of the router's PS admission stage).
3. **Completion** — finished trajectories are scored, collected per group, and
   a completed group is committed with ``occupy_rollout_instance_request``;
   optional group post-processing (DAPO dynamic-sampling filter) drops
   zero-variance groups and replaces them.
4. **Readiness** — when a buffer turns READY the PS runs its staleness aborts
   (``handle_ready_buffer``); aborted requests are forwarded to the instances.
5. **Consumption** — the trainer takes the trajectories of a READY buffer.
6. **Retry** — groups that lost too many members are replaced by fresh prompts.
7. **Failure recovery** — a trajectory that stops on an error or a timeout
   (:mod:`.terminate`) is retried up to ``rollout.agent.retry_limit``
   attempts; if it still fails, ``notify_group_failed`` aborts its siblings
   and refills the lost buffer slot with a fresh prompt
   (reference ``manager.py:543`` ``notify_group_failed``, ``:398``
   ``_retry_data``, ``worker.py:392-470``).  Requests running longer than
   ``rollout.agent.trajectory_timeout_s`` are aborted as trajectory
   timeouts.
8. **Waiting buffers** — when the trainer has waited on a buffer for
   ``proactive_filter_strategy.patience_s`` and at most ``threshold``
   entries are missing, ``handle_waiting_buffer`` either (``retry``) aborts
   the buffer's reservations, moves occupied entries of later buffers into it
   and dispatches fresh prompts for the aborted ones, or (``truncate``)
   aborts the reservations and releases the buffer with the entries it has
   (reference ``manager.py:1327``).

All methods are thread-safe (one lock), so the same object serves in-process
callers and the RPC server threads of remote rollout instances.
"""

from __future__ import annotations

import threading
import time
from collections import deque
from dataclasses import dataclass, field

from ..config import redundant_settings
from ..ps import BufferStatus, PSManager, RequestStatus
from ..rollout.engine import GenRequest, RequestOutput, SamplingParams
from ..trainer.batch import Trajectory
from .data import DataProcessor
from .terminate import TerminateReason, reason_of_exception, reason_of_finish


@dataclass
class _Group:
    uid: int
    prompt_ids: list
    meta: dict
    request_ids: list
    done: dict = field(default_factory=dict)      # request_id -> Trajectory
    dropped: set = field(default_factory=set)
    committed: bool = False


class AgentLoopManager:
    def __init__(self, cfg, ps: PSManager, data: DataProcessor, reward, initial_ps_version: int = 0,
                 agent_loop=None):
        from .loops import build_agent_loop
        self.cfg = cfg
        vocab = data.src.vocab if hasattr(data.src, "vocab") else 1024
        self.loop = agent_loop if agent_loop is not None else build_agent_loop(cfg, vocab,
                                                                               getattr(data, "tokenizer", None))
        self.ps = ps
        self.data = data
        self.reward = reward
        self.rollout_n, self.alg_rollout_n, self.entries, self.ready_entries = redundant_settings(cfg)
        self.staleness = int(cfg.psrl.staleness)
        self.max_ahead = int(cfg.psrl.get("max_dispatch_ahead", 5))
        self.buffer_size = self.entries * self.rollout_n       # trajectories per buffer
        self.initial_ps_version = int(initial_ps_version)
        self.request_counter = 0
        self.lock = threading.RLock()
        self.queue: deque[GenRequest] = deque()
        self.groups: dict[int, _Group] = {}
        self.store: dict[int, list[Trajectory]] = {}           # committed groups by prompt id
        self.pending_aborts: dict = {}                         # instance_id -> set(request ids)
        self.rp = cfg.rollout
        self.max_response = int(cfg.rollout.max_response_length)
        gp = cfg.psrl.group_post_process
        self.group_filter = gp.name if gp.enable else "no_filter"
        self.filter_metric = gp.get("metric", "acc")
        self.stats = {"dispatched_groups": 0, "completed_trajs": 0, "dropped_trajs": 0, "filtered_groups": 0,
                      "retried_groups": 0, "aborted_requests": 0, "retried_trajs": 0, "failed_groups": 0,
                      "timed_out_trajs": 0, "waiting_buffer_moves": 0, "truncated_buffers": 0}
        ag = cfg.rollout.get("agent", None) or {}
        self.retry_limit = max(1, int(ag.get("retry_limit", 1)))
        self.trajectory_timeout_s = ag.get("trajectory_timeout_s", None)
        self.manager_retry_on_error = bool(cfg.psrl.agentic_rl.get("manager_retry_on_error", True))
        pf = cfg.psrl.rollout_coordination.proactive_filter_strategy
        self.filter_method = pf.get("method", None)
        self.filter_threshold = int(pf.get("threshold", 0))
        self.filter_patience_s = float(pf.get("patience_s", 5.0))
        self.attempts: dict[int, int] = {}          # request id -> failed attempts so far
        self.failed_groups: set[int] = set()
        self.started_at: dict[int, float] = {}      # request id -> time handed to an instance
        self.timed_out: set[int] = set()
        self.last_error: str | None = None
        self.migration_target: dict[int, tuple] = {}   # request id -> instance it is moving to
        ps.on_abort_rollout = self._on_abort_rollout

    # ------------------------------------------------------------ dispatch
    def expected_ps_version(self) -> int:
        eff = min(self.staleness, self.max_ahead)
        return self.initial_ps_version + max(self.request_counter - eff * self.buffer_size, 0) // self.buffer_size

    def _dispatch_group(self) -> None:
        item = self.data.next_group()
        uid = item.uid
        rids = [uid * self.rollout_n + j for j in range(self.rollout_n)]
        self.ps.add_request(rids, status=RequestStatus.PENDING)
        self.ps.update_request_status(rids, RequestStatus.RUNNING)
        meta = dict(item.meta)
        if item.answer is not None:
            meta["answer"] = item.answer
        self.groups[uid] = _Group(uid, item.prompt_ids, meta, rids)
        for j, rid in enumerate(rids):
            mt = item.response_lens[j] if item.response_lens else self.max_response
            params = SamplingParams(temperature=float(self.rp.temperature), top_p=float(self.rp.top_p),
                                    top_k=int(self.rp.top_k), max_tokens=int(mt),
                                    ignore_eos=bool(self.rp.ignore_eos), seed=rid * 7919 + 17)
            self.queue.append(GenRequest(rid, item.prompt_ids, params, -1, {"uid": uid, "max_tokens": int(mt), **meta}))
        self.request_counter += self.rollout_n
        self.stats["dispatched_groups"] += 1

    def fill(self, max_queued: int | None = None) -> int:
        """Release prompt groups allowed by the dispatch-ahead bound."""
        with self.lock:
            cap = max_queued if max_queued is not None else 4 * self.buffer_size
            ps_v = self.ps.get_ps_model_version()
            n = 0
            while len(self.queue) < cap and self.expected_ps_version() <= ps_v:
                self._dispatch_group()
                n += 1
            return n

    def take_work(self, instance_id, instance_version: int, max_n: int, accept=None) -> list[GenRequest]:
        """Admission: reserve each request at the instance's version and hand it
        out.  ``accept(req) -> bool`` (the router's pull-mode policy) may pass
        a request over for another instance; at most ``4 * max_n`` requests
        are looked at per call."""
        with self.lock:
            self.fill()
            self._check_trajectory_timeouts()
            out: list[GenRequest] = []
            held: list[GenRequest] = []       # migrating elsewhere, or routed to another instance
            looked = 0
            while self.queue and len(out) < max_n and looked < 4 * max(1, max_n):
                looked += 1
                req = self.queue[0]
                rid = req.request_id
                tgt = self.migration_target.get(rid)
                if tgt is not None and tgt != instance_id:
                    held.append(self.queue.popleft())
                    continue
                if tgt is None and accept is not None and not accept(req):
                    held.append(self.queue.popleft())
                    self.stats["routed_elsewhere"] = self.stats.get("routed_elsewhere", 0) + 1
                    continue
                self.migration_target.pop(rid, None)
                if self.ps.check_aborted_requests(rid, remove=True):
                    self.queue.popleft()
                    self._member_dropped(rid)
                    continue
                if not self.ps.can_reserve_request(rid, [instance_version])[0]:
                    break
                self.queue.popleft()
                self.ps.reserve_rollout_instance_requests(instance_id, rid, instance_version)
                self.ps.update_request_status(rid, RequestStatus.ROLLOUT_RUNNING, model_version=instance_version,
                                              rollout_instance_id=instance_id)
                # a fresh or partially generated request (re)starts at the instance's
                # version (partial rollouts are promoted); a later turn of a
                # multi-turn session keeps the version pinned at its first turn
                if req.meta.get("turn", 0) == 0:
                    req.version_tag = instance_version
                    if req.prev_output_ids:
                        self.ps.update_request_version_tag(rid, instance_version)
                self.started_at.setdefault(rid, time.monotonic())
                out.append(req)
            self.queue.extendleft(reversed(held))
            return out

    def migrate(self, src, dst, n: int) -> int:
        """Move up to ``n`` requests running on instance ``src`` to ``dst``
        (load-balanced migration, reference ``sync_and_migrate/greedy.py``): the
        source is told to interrupt them; their partial outputs come back as
        ``abort`` results, are re-queued with the tokens generated so far and
        are handed only to ``dst``, which resumes them after a re-prefill."""
        with self.lock:
            running = sorted(r for r in self.ps.get_dispatched_requests_of_instance(src)
                             if self.ps.get_request_status(r)[0] is RequestStatus.ROLLOUT_RUNNING)
            pending = self.pending_aborts.get(src, set())
            pick = [r for r in running if r not in pending and r not in self.timed_out][-int(n):] if n > 0 else []
            for rid in pick:
                self.migration_target[rid] = dst
            if pick:
                self.pending_aborts.setdefault(src, set()).update(pick)
                self.stats["migrated_requests"] = self.stats.get("migrated_requests", 0) + len(pick)
            return len(pick)

    def _check_trajectory_timeouts(self) -> None:
        """Abort requests that have run longer than the trajectory timeout; their
        abort output comes back as a TRAJECTORY_TIMEOUT failure."""
        if not self.trajectory_timeout_s:
            return
        now = time.monotonic()
        late = [r for r, t in self.started_at.items() if now - t > float(self.trajectory_timeout_s)
                and r not in self.timed_out]
        if not late:
            return
        live = [r for r in late if self.ps.has_request(r)]
        by_inst = self.ps.classify_requests_in_instance(live) if live else {}
        for inst, rids in by_inst.items():
            self.pending_aborts.setdefault(inst, set()).update(rids)
        for rid in late:
            self.timed_out.add(rid)
            self.stats["timed_out_trajs"] += 1

    # ---------------------------------------------------------- completion
    def on_complete(self, outputs: list[RequestOutput], instance_id=None) -> None:
        with self.lock:
            for o in outputs:
                self._complete_one(o, instance_id)
            turns = self._turn_records()
            if turns is not None:
                for o in outputs:
                    turns.from_output(o)
                if len(turns.data) >= 256:
                    turns.flush()

    def _turn_records(self):
        """Per-request turn records (``trainer.turn_records_path``, JSON lines;
        written in batches of 256 requests), or None."""
        if not hasattr(self, "_turns"):
            path = self.cfg.trainer.get("turn_records_path", None) if hasattr(self.cfg, "trainer") else None
            from ..utils.profiling import TurnProfilingCollector
            self._turns = TurnProfilingCollector(str(path)) if path else None
        return self._turns

    def flush_turn_records(self) -> int:
        t = self._turn_records()
        return t.flush() if t is not None else 0

    def _complete_one(self, o: RequestOutput, instance_id=None) -> None:
        rid = o.request_id
        if rid in self.timed_out:
            self.timed_out.discard(rid)
            self._on_failure(o, TerminateReason.TRAJECTORY_TIMEOUT, "trajectory timeout")
            return
        reason = reason_of_finish(o.finish_reason)
        if reason.needs_worker_retry():
            self._on_failure(o, reason, f"engine finish reason {o.finish_reason!r}")
            return
        try:
            self._finish_one(o, instance_id)
        except Exception as exc:  # environment, tool or reward failure
            self._on_failure(o, reason_of_exception(exc), f"{type(exc).__name__}: {exc}")

    def _on_failure(self, o: RequestOutput, reason: TerminateReason, why: str) -> None:
        """A trajectory stopped without usable data: retry it, or give up its
        group and refill the slot (worker retry, then manager retry)."""
        rid = o.request_id
        uid = rid // self.rollout_n
        self.started_at.pop(rid, None)
        self.last_error = f"request {rid}: {reason.value} ({why})"
        if getattr(self.loop, "multi_turn", False):
            self.loop.drop(rid)
        g = self.groups.get(uid)
        if g is None or g.committed:
            return
        n = self.attempts.get(rid, 0) + 1
        self.attempts[rid] = n
        if reason.needs_worker_retry() and n < self.retry_limit and not self.ps.check_aborted_requests(rid):
            # try the trajectory again from its prompt, on whichever instance takes it
            meta = {k: v for k, v in o.meta.items() if k not in ("turn",)}
            self.queue.appendleft(GenRequest(rid, list(g.prompt_ids), self._params_of(o), -1, meta))
            self.stats["retried_trajs"] += 1
            return
        if reason.needs_manager_retry():
            if not self.manager_retry_on_error:
                raise RuntimeError(f"rollout of request {rid} failed after {n} attempt(s): {self.last_error}; "
                                   "set psrl.agentic_rl.manager_retry_on_error=true to recover")
            self.notify_group_failed(uid, rid, reason)
            return
        self._member_dropped(rid)

    def notify_group_failed(self, uid: int, failed_request_id: int, reason: TerminateReason | None = None) -> None:
        """A member of group ``uid`` failed for good: abort its siblings, drop the
        group and dispatch one fresh prompt in its place (once per group)."""
        with self.lock:
            if uid in self.failed_groups:
                return
            self.failed_groups.add(uid)
            g = self.groups.get(uid)
            if g is None or g.committed:
                return
            self.stats["failed_groups"] += 1
            self._retire_group(g, replace=True)

    def _finish_one(self, o: RequestOutput, instance_id=None) -> None:
        rid = o.request_id
        uid = rid // self.rollout_n
        g = self.groups.get(uid)
        if o.finish_reason == "abort":
            # interrupted for migration: back to the queue with its partial output
            if g is not None and not self.ps.check_aborted_requests(rid, remove=False):
                self.queue.appendleft(GenRequest(rid, o.prompt_ids, self._params_of(o), o.version_tag, o.meta,
                                                 o.output_ids, o.logprobs, o.versions))
            return
        if g is None:
            return
        st = self.ps.get_request_status(rid)[0] if self.ps.has_request(rid) else None
        if st is None:
            self._member_dropped(rid)
            return
        if self.loop.multi_turn:
            nxt = self.loop.on_turn_complete(o, instance_id)
            if nxt is not None:
                self.queue.appendleft(nxt)       # next turn, sticky to this instance
                return
        sample = self.loop.finalize(o)
        # the engine promotes the tag when it re-prefills after a weight update
        self.ps.update_request_version_tag(rid, o.version_tag)
        if not self.ps.update_request_status(rid, RequestStatus.ROLLOUT_COMPLETED, model_version=o.version_tag):
            self._member_dropped(rid)
            return
        traj = Trajectory(uid=uid, request_id=rid, prompt_ids=sample["prompt_ids"], response_ids=sample["response_ids"],
                          rollout_logprobs=sample["logprobs"], versions=sample["versions"], version_tag=o.version_tag,
                          response_mask=sample["response_mask"], meta={**o.meta, "turns": sample["turns"],
                                                                      "env_info": sample.get("env_info") or {}})
        self.ps.update_request_status(rid, RequestStatus.REWARD_RUNNING)
        sc = self.reward.score(traj)
        traj.reward = float(sc["score"])
        traj.meta["reward_extra"] = sc
        if not self.ps.update_request_status(rid, RequestStatus.COMPLETED):
            self._member_dropped(rid)
            return
        g.done[rid] = traj
        self.started_at.pop(rid, None)
        self.stats["completed_trajs"] += 1
        self._maybe_commit(g)

    def _params_of(self, o: RequestOutput) -> SamplingParams:
        rp = self.rp
        mt = o.meta.get("max_tokens", None)
        return SamplingParams(temperature=float(rp.temperature), top_p=float(rp.top_p), top_k=int(rp.top_k),
                              max_tokens=int(mt or (len(o.output_ids) + self.max_response)),
                              ignore_eos=bool(rp.ignore_eos), seed=o.request_id * 7919 + 17)

    def _member_dropped(self, rid: int) -> None:
        if getattr(self.loop, "multi_turn", False):
            self.loop.drop(rid)
        uid = rid // self.rollout_n
        g = self.groups.get(uid)
        if g is None:
            return
        g.dropped.add(rid)
        self.stats["dropped_trajs"] += 1
        self._maybe_commit(g)

    def _maybe_commit(self, g: _Group) -> None:
        if g.committed:
            return
        live = len(g.request_ids) - len(g.dropped)
        if live < self.alg_rollout_n:
            # the group can no longer be completed: drop it and replace the prompt
            self._retire_group(g, replace=True)
            return
        if len(g.done) < self.alg_rollout_n:
            return
        chosen = sorted(g.done)[: self.alg_rollout_n] if len(g.done) > self.alg_rollout_n else sorted(g.done)
        trajs = [g.done[r] for r in chosen]
        if self.group_filter == "dynamic_sampling_filter":
            vals = [t.meta["reward_extra"].get(self.filter_metric, t.reward) for t in trajs]
            if len(set(vals)) <= 1 and len(vals) > 1:
                self.stats["filtered_groups"] += 1
                self._retire_group(g, replace=True)
                return
        # redundant members still in flight are no longer needed
        extra = [r for r in g.request_ids if r not in g.done and r not in g.dropped]
        if extra:
            self.ps.abort_requests(extra, abort_group=False)
        bid, occ, entry = self.ps.occupy_rollout_instance_request(g.uid, chosen)
        g.committed = True
        self.groups.pop(g.uid, None)
        if bid is None:
            self._retire_group(g, replace=True)
            return
        self.store[g.uid] = trajs
        status = self.ps.get_buffer_status(bid)
        if status in (BufferStatus.READY, BufferStatus.READY_WITH_CAPACITY):
            aborted = self.ps.handle_ready_buffer(bid)
            self.stats["aborted_requests"] += len(aborted)

    def _retire_group(self, g: _Group, replace: bool) -> None:
        g.committed = True
        self.groups.pop(g.uid, None)
        alive = [r for r in g.request_ids if self.ps.has_request(r)]
        if alive:
            self.ps.abort_requests(alive, abort_group=True)
        # purge queued members of the group
        self.queue = deque(r for r in self.queue if r.request_id // self.rollout_n != g.uid)
        if replace:
            self.stats["retried_groups"] += 1
            self._dispatch_group()

    def _on_abort_rollout(self, instance_to_ids: dict) -> None:
        for inst, ids in instance_to_ids.items():
            self.pending_aborts.setdefault(inst, set()).update(ids)

    def take_aborts(self, instance_id) -> list[int]:
        with self.lock:
            return sorted(self.pending_aborts.pop(instance_id, set()))

    # ---------------------------------------------------- waiting buffers
    def handle_waiting_buffer(self, buffer_id: int) -> bool:
        """The trainer has waited on ``buffer_id`` for the patience window.  With
        at most ``threshold`` entries missing, apply the configured strategy;
        returns True if the buffer changed."""
        if self.filter_method not in ("retry", "truncate"):
            return False
        from ..ps import EntryCategory
        with self.lock:
            self.ps.ensure_train_buffer_exists(buffer_id)
            inv = self.ps.staleness_inventory
            buf = inv.buffers.get(buffer_id)
            if buf is None:
                return False
            occupied = min(buf.get_first_non_occupied(), buf.ready_num_entries)
            gap = buf.ready_num_entries - occupied
            if gap <= 0 or gap > self.filter_threshold:
                return False
            if self.filter_method == "retry":
                donors = []
                for other in sorted(inv.buffers, reverse=True):
                    if other <= buffer_id:
                        break
                    donors += [e.entry_info for e in inv.buffers[other].entries
                               if e.category is EntryCategory.OCCUPIED]
                if len(donors) < gap:
                    return False
                n_aborted = self._abort_buffer_reservations(buffer_id)
                inv.move_occupied_entries(donors[:gap], buffer_id)
                self.stats["waiting_buffer_moves"] += gap
                for _ in range(n_aborted):
                    self.stats["retried_groups"] += 1
                    self._dispatch_group()
            else:
                self._abort_buffer_reservations(buffer_id)
                # release the buffer with the committed entries it holds
                first_free = buf.get_first_non_occupied()
                buf.ready_num_entries = max(1, first_free)
                self.stats["truncated_buffers"] += 1
            if self.ps.get_buffer_status(buffer_id) in (BufferStatus.READY, BufferStatus.READY_WITH_CAPACITY):
                self.stats["aborted_requests"] += len(self.ps.handle_ready_buffer(buffer_id))
            return True

    def _abort_buffer_reservations(self, buffer_id: int) -> int:
        """Abort every reserved (in-flight) group of a buffer and forget it here;
        returns how many groups were aborted."""
        buf = self.ps.staleness_inventory.buffers[buffer_id]
        pids = [buf.entries[e].entry_info.prompt_id for e in buf.get_reserved_entry_ids()]
        n, _ = self.ps.abort_reserved_requests(buffer_id)
        for pid in pids:
            g = self.groups.get(pid)
            if g is not None:
                self._retire_group(g, replace=False)
        return n

    # ------------------------------------------------------------- trainer
    def buffer_ready(self, buffer_id: int) -> bool:
        with self.lock:
            self.ps.ensure_train_buffer_exists(buffer_id)
            st = self.ps.get_buffer_status(buffer_id)
            return st in (BufferStatus.READY, BufferStatus.READY_WITH_CAPACITY)

    def occupied_prefix(self, buffer_id: int) -> int:
        """Number of committed (OCCUPIED) entries at the head of a buffer's training region."""
        with self.lock:
            self.ps.ensure_train_buffer_exists(buffer_id)
            buf = self.ps.staleness_inventory.buffers.get(buffer_id)
            return 0 if buf is None else min(buf.get_first_non_occupied(), buf.ready_num_entries)

    def peek(self, buffer_id: int, lo: int, hi: int) -> list[Trajectory]:
        """Trajectories of entries [lo, hi) of a buffer without consuming them
        (the objects are shared with what ``consume`` later returns)."""
        with self.lock:
            buf = self.ps.staleness_inventory.buffers[buffer_id]
            out: list[Trajectory] = []
            for e in buf.entries[lo:hi]:
                info = e.entry_info
                keep = set(info.get_all_request_ids(self.rollout_n))
                out.extend(t for t in self.store.get(info.prompt_id, []) if t.request_id in keep)
            return out

    def consume(self, buffer_id: int) -> list[Trajectory]:
        with self.lock:
            entries = self.ps.consume_buffer(buffer_id)
            out: list[Trajectory] = []
            for e in entries:
                trajs = self.store.pop(e.prompt_id, [])
                keep = set(e.get_all_request_ids(self.rollout_n))
                out.extend(t for t in trajs if t.request_id in keep)
            return out

    def snapshot(self) -> dict:
        with self.lock:
            return {"queue": len(self.queue), "open_groups": len(self.groups), "stored_groups": len(self.store),
                    "request_counter": self.request_counter, "expected_ps_version": self.expected_ps_version(),
                    **self.stats}
