"""Request lifecycle tracking for the Parameter Server.

Lifecycle states and abort semantics follow the reference
(``psrl/workers/ps/request_status_tracker.py:33-216,340-450``):

* every request (one trajectory of a prompt group; ``request_id = prompt_id *
  rollout_n + request_idx``) moves PENDING → RUNNING → ROLLOUT_* → REWARD_* →
  COMPLETED;
* an abort only *marks* a request; the next status update of that request
  returns ``False`` and drops it, so racing producers learn about it lazily;
* a request whose version fell below the running minimum version is stale and
  its update is refused;
* payloads already committed to the sample store (ROLLOUT_COMPLETED,
  REWARD_RUNNING, REWARD_COMPLETED) are cleared from the store on abort.

Side effects of aborts on other components (stop generation, cancel reward,
delete stored samples) are delivered through plain callbacks registered by the
runtime instead of actor handles.
"""

from __future__ import annotations

import enum
import threading
from collections import defaultdict
from typing import Callable, Iterable

from .staleness import INVALID_ROLLOUT_INSTANCE_ID, EntryInfo, state_locked


class RequestStatus(enum.Enum):
    PENDING = enum.auto()
    RUNNING = enum.auto()
    ROLLOUT_ROUTING = enum.auto()
    ROLLOUT_DISPATCHED = enum.auto()
    ROLLOUT_RUNNING = enum.auto()
    ROLLOUT_INTERRUPTED = enum.auto()
    ROLLOUT_COMPLETED = enum.auto()
    REWARD_RUNNING = enum.auto()
    REWARD_COMPLETED = enum.auto()
    COMPLETED = enum.auto()


# Alias with the reference's public name.
PSRL_RequestStatus = RequestStatus

STORE_COMMITTED_STATUSES = frozenset(
    {RequestStatus.ROLLOUT_COMPLETED, RequestStatus.REWARD_RUNNING, RequestStatus.REWARD_COMPLETED}
)


def _listify(x, n: int | None = None) -> list:
    if isinstance(x, list):
        return x
    return [x] * (n if n is not None else 1)


class RequestStatusTracker:
    def __init__(self, rollout_n: int, alg_rollout_n: int | None = None, val_rollout_n: int = 1):
        self._state_lock = threading.RLock()
        self.rollout_n = int(rollout_n)
        self.alg_rollout_n = int(alg_rollout_n or rollout_n)
        self.val_rollout_n = int(val_rollout_n)
        self._status: dict[int, RequestStatus] = {}
        self._infos: dict[int, EntryInfo] = {}
        self._by_status: dict[RequestStatus, set[int]] = {s: set() for s in RequestStatus}
        self._abort_request_ids: set[int] = set()
        self._running_min_version = 0
        # Callbacks: (instance_id -> [request ids]) for rollout, ids for reward, ids for the store.
        self.on_abort_rollout: Callable[[dict], None] | None = None
        self.on_abort_reward: Callable[[list[int]], None] | None = None
        self.on_clear_store: Callable[[list[int], bool], None] | None = None

    # ------------------------------------------------------------- add/remove
    @state_locked
    def add_request(self, request_id, rollout_instance_id=INVALID_ROLLOUT_INSTANCE_ID, model_version=-1,
                    status=RequestStatus.PENDING, is_validate=False) -> None:
        ids = _listify(request_id)
        n = len(ids)
        insts = rollout_instance_id if isinstance(rollout_instance_id, list) else [rollout_instance_id] * n
        vers = _listify(model_version, n)
        stats = _listify(status, n)
        vals = _listify(is_validate, n)
        for rid, inst, ver, st, val in zip(ids, insts, vers, stats, vals):
            rn = self.val_rollout_n if val else self.rollout_n
            self._infos[rid] = EntryInfo(inst, rid // rn, rid % rn, ver, 1, val)
            self._status[rid] = st
            self._by_status[st].add(rid)

    @state_locked
    def remove_request(self, request_id) -> None:
        for rid in _listify(request_id):
            st = self._status.pop(rid, None)
            if st is not None:
                self._by_status[st].discard(rid)
            self._infos.pop(rid, None)
            self._abort_request_ids.discard(rid)

    @state_locked
    def remove_train_ready_request(self, request_id) -> None:
        for rid in _listify(request_id):
            if self._status.get(rid) is not RequestStatus.COMPLETED:
                raise AssertionError(f"request {rid} is not COMPLETED (status {self._status.get(rid)})")
            if rid in self._abort_request_ids:
                raise AssertionError(f"request {rid} is marked aborted")
        self.remove_request(request_id)

    @state_locked
    def clear_request_status_manager(self) -> None:
        self._status.clear()
        self._infos.clear()
        self._abort_request_ids.clear()
        for s in self._by_status.values():
            s.clear()

    # ----------------------------------------------------------------- status
    def _check_aborted_request(self, request_id: int, remove: bool = True) -> bool:
        if request_id in self._abort_request_ids:
            if remove:
                self.remove_request(request_id)
            return True
        return request_id not in self._status

    @state_locked
    def update_request_status(self, request_id, status, model_version=-1,
                              rollout_instance_id=INVALID_ROLLOUT_INSTANCE_ID, is_validate=False):
        """Set statuses; returns per-request success (False = aborted or stale)."""
        ids = _listify(request_id)
        n = len(ids)
        stats = _listify(status, n)
        vers = _listify(model_version, n)
        insts = rollout_instance_id if isinstance(rollout_instance_id, list) else [rollout_instance_id] * n
        ok = [True] * n
        stale_committed: list[int] = []
        for i, rid in enumerate(ids):
            if self._check_aborted_request(rid, remove=True):
                ok[i] = False
                continue
            info = self._infos[rid]
            if insts[i] != INVALID_ROLLOUT_INSTANCE_ID:
                info.rollout_instance_id[0] = insts[i]
            if vers[i] != -1:
                info.model_version[0] = int(vers[i])
            v = info.model_version[0]
            if not is_validate and v != -1 and v < self._running_min_version:
                ok[i] = False
                if self._status[rid] in STORE_COMMITTED_STATUSES:
                    stale_committed.append(rid)
                continue
            old = self._status[rid]
            self._by_status[old].discard(rid)
            self._status[rid] = stats[i]
            self._by_status[stats[i]].add(rid)
        if stale_committed and self.on_clear_store:
            self.on_clear_store(stale_committed, is_validate)
        return ok[0] if n == 1 and not isinstance(request_id, list) else ok

    @state_locked
    def get_request_status(self, request_id) -> list[RequestStatus]:
        ids = _listify(request_id)
        out = [self._status.get(r) for r in ids]
        if any(s is None for s in out):
            raise KeyError(f"unknown request ids in {ids}")
        return out

    def has_request(self, request_id: int) -> bool:
        with self._state_lock:
            return request_id in self._status

    @state_locked
    def get_all_request_statuses(self) -> dict[int, RequestStatus]:
        return dict(self._status)

    @state_locked
    def get_requests_by_status(self, status: RequestStatus) -> set[int]:
        return set(self._by_status[status])

    @state_locked
    def get_request_info(self, request_id):
        if isinstance(request_id, list):
            return [self._infos.get(r) for r in request_id]
        return self._infos.get(request_id)

    @state_locked
    def update_request_version(self, request_id, new_version: int) -> None:
        for rid in _listify(request_id):
            if rid in self._infos:
                self._infos[rid].model_version[0] = int(new_version)

    @state_locked
    def update_request_instance(self, request_id, new_instance) -> None:
        for rid in _listify(request_id):
            if rid in self._infos:
                self._infos[rid].rollout_instance_id[0] = new_instance

    def set_running_min_version(self, version: int) -> None:
        with self._state_lock:
            self._running_min_version = int(version)

    # -------------------------------------------------------------- queries
    @state_locked
    def classify_requests_in_status(self, request_ids) -> dict[RequestStatus, list[int]]:
        out: dict[RequestStatus, list[int]] = defaultdict(list)
        for rid in _listify(request_ids):
            st = self._status.get(rid)
            if st is not None:
                out[st].append(rid)
        return dict(out)

    @state_locked
    def classify_requests_in_instance(self, request_ids) -> dict:
        out: dict = defaultdict(list)
        for rid in _listify(request_ids):
            info = self._infos.get(rid)
            if info is not None:
                out[info.rollout_instance_id[0]].append(rid)
        return dict(out)

    @state_locked
    def get_requests_ids_of_version(self, version: int) -> set[int]:
        return {rid for rid, info in self._infos.items() if info.model_version[0] == version}

    @state_locked
    def get_dispatched_requests_of_instance(self, instance_id) -> set[int]:
        return {rid for rid, info in self._infos.items() if info.rollout_instance_id[0] == instance_id}

    @state_locked
    def get_requests_of_abort_version(self, version: int) -> set[int]:
        """Unfinished training requests whose version is <= ``version``."""
        live = (RequestStatus.COMPLETED,)
        return {
            rid for rid, info in self._infos.items()
            if not info.is_validate and 0 <= info.model_version[0] <= version and self._status[rid] not in live
        }

    @state_locked
    def get_recorded_child_requests(self, parent_id, is_validate: bool = False) -> set[int]:
        rn = self.val_rollout_n if is_validate else self.rollout_n
        pids = set(_listify(parent_id))
        return {rid for rid in self._infos if rid // rn in pids}

    # ---------------------------------------------------------------- abort
    @state_locked
    def _abort_requests(self, request_ids, blocking: bool = False) -> None:
        ids = {r for r in _listify(request_ids) if r in self._status}
        self._abort_request_ids |= ids
        by_status = self.classify_requests_in_status(list(ids))
        rollout_ids = by_status.get(RequestStatus.ROLLOUT_RUNNING, []) + by_status.get(
            RequestStatus.ROLLOUT_DISPATCHED, [])
        reward_ids = by_status.get(RequestStatus.REWARD_RUNNING, [])
        completed = by_status.get(RequestStatus.COMPLETED, [])
        stored = [r for s in STORE_COMMITTED_STATUSES for r in by_status.get(s, [])]
        if rollout_ids and self.on_abort_rollout:
            self.on_abort_rollout(self.classify_requests_in_instance(rollout_ids))
        if reward_ids and self.on_abort_reward:
            self.on_abort_reward(reward_ids)
        if stored and self.on_clear_store:
            self.on_clear_store(stored, False)
        # A completed request has nothing in flight: drop it now.
        for rid in completed:
            self.remove_request(rid)

    # -------------------------------------------------- data of in-flight reqs
    def check_abort_set(self) -> set[int]:
        with self._state_lock:
            return set(self._abort_request_ids)


__all__ = ["PSRL_RequestStatus", "RequestStatus", "RequestStatusTracker", "STORE_COMMITTED_STATUSES"]
