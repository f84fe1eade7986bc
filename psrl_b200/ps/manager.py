"""The Parameter Server manager: model version, staleness inventories, admission
(Reserve), completion (Occupy), consumption and staleness aborts, plus the
push/pull lock that orders weight publication against weight reads.

Reference behaviour: ``psrl/workers/ps/ps_manager.py`` (``ModelStore`` :42,
``can_reserve_request`` :385, ``get_reserve_indicator`` :456,
``reserve_rollout_instance_requests`` :506, ``abort_requests`` :623,
``_abort_after_buffer_ready`` :730, ``occupy_rollout_instance_request`` :835,
``maybe_delete_buffer`` :360, locks :1170-1207, push/pull :1226-1380,
``init_model_version_for_resume`` :1209).

B200 design differences:

* The manager is a plain in-process object (thread-safe through a re-entrant
  lock).  Other processes reach it through :mod:`psrl_b200.utils.rpc`, which
  replaces both Ray actor calls and the gRPC surface the Rust router used.
* The weight store is not a pinned-CPU NIXL buffer: with ``ps_mode=hbm`` the
  published weights live in trainer HBM (see
  :mod:`psrl_b200.parallel.weight_sync`); the manager only tracks the version
  and a handle describing where the current weights are.
"""

from __future__ import annotations

import threading
import time
from collections.abc import Callable
from dataclasses import dataclass, field
from typing import Any

from .request_tracker import RequestStatus, RequestStatusTracker
from .staleness import (
    INVALID_ROLLOUT_INSTANCE_ID,
    BufferStatus,
    EntryCategory,
    EntryInfo,
    StalenessInventory,
    state_locked,
)


@dataclass
class ModelStore:
    """Published model version plus an opaque handle to its storage."""

    version_tag: int = 0
    state: Any = None        # cpu/cpu_ref: state dict; hbm: WeightStoreHandle
    push_time: float = 0.0


@dataclass
class RolloutInstanceStatus:
    version_tag: int = 0
    meta: dict = field(default_factory=dict)


class PSManager(RequestStatusTracker):
    def __init__(self, staleness: int, staleness_buffer_entries: int, rollout_n: int,
                 redundant_rollout: dict | None = None, val_rollout_n: int = 1):
        rr = redundant_rollout or {}
        if rr.get("enable"):
            rn, alg_rn = int(rr["redundant_rollout_n"]), int(rr["alg_rollout_n"])
            entries, ready = int(rr["redundant_global_batch_size"]), int(rr["alg_global_batch_size"])
        else:
            rn = alg_rn = int(rollout_n)
            entries = ready = int(staleness_buffer_entries)
        super().__init__(rn, alg_rn, val_rollout_n)
        self.staleness = int(staleness)
        self.entries_per_buffer = entries
        self.ready_entries_per_buffer = ready
        self.staleness_inventory = StalenessInventory(entries, ready, self.staleness, rn)
        self.val_staleness_inventory = StalenessInventory(ready, ready, None, val_rollout_n, is_validate=True)
        self.model_store = ModelStore(version_tag=0)
        self.rollout_instance_tracker: dict[Any, RolloutInstanceStatus] = {}
        self.check_abort_versions: set[int] = set()
        self.max_aborted_version = -1
        # push/pull reader-writer lock
        self._rw = threading.Condition()
        self._exclusive_push_locked = False
        self._shared_pull_count = 0
        # listeners
        self.on_version_published: list[Callable[[int], None]] = []
        self.on_buffer_ready: list[Callable[[int], None]] = []

    @classmethod
    def from_config(cls, cfg) -> "PSManager":
        p = cfg.psrl
        rr = p.rollout_coordination.redundant_rollout
        return cls(p.staleness, p.staleness_buffer_entries, p.rollout_n,
                   redundant_rollout=rr.to_dict() if hasattr(rr, "to_dict") else dict(rr),
                   val_rollout_n=p.val_rollout_n)

    def _inv(self, is_validate: bool) -> StalenessInventory:
        return self.val_staleness_inventory if is_validate else self.staleness_inventory

    def _rn(self, is_validate: bool) -> int:
        return self.val_rollout_n if is_validate else self.rollout_n

    # ----------------------------------------------------- rollout instances
    @state_locked
    def register_rollout_instance(self, instance_id, version_tag: int | None = None, **meta) -> None:
        v = self.model_store.version_tag if version_tag is None else int(version_tag)
        self.rollout_instance_tracker[instance_id] = RolloutInstanceStatus(v, dict(meta))

    @state_locked
    def get_rollout_instance_model_version(self, instance_id) -> int:
        return self.rollout_instance_tracker[instance_id].version_tag

    @state_locked
    def set_rollout_instance_model_version(self, instance_id, version: int) -> None:
        self.rollout_instance_tracker.setdefault(instance_id, RolloutInstanceStatus()).version_tag = int(version)
        self._refresh_running_min_version()

    @state_locked
    def get_all_rollout_instance_model_versions(self) -> dict:
        return {k: v.version_tag for k, v in self.rollout_instance_tracker.items()}

    def _refresh_running_min_version(self) -> None:
        # A request older than the oldest version any live buffer admits is stale.
        self.set_running_min_version(max(0, self.model_store.version_tag - self.staleness))

    # ------------------------------------------------------------ versions
    @state_locked
    def get_ps_model_version(self, debug_info: str = "") -> int:
        return self.model_store.version_tag

    @state_locked
    def init_model_version_for_resume(self, global_step: int) -> None:
        """Resuming at trainer step ``global_step`` means version ``global_step - 1``
        was the last published one; buffers below it no longer exist."""
        v = max(0, int(global_step) - 1)
        self.model_store.version_tag = v
        inv = self.staleness_inventory
        if inv.buffer_id < v:
            inv.buffer_id = v
        self._refresh_running_min_version()

    # ---------------------------------------------------------- admission
    @state_locked
    def can_reserve_request(self, request_idx, model_versions: list[int], without_new_reserve_entry: bool = False,
                            is_validate=False):
        single = not isinstance(request_idx, list)
        ids = [request_idx] if single else list(request_idx)
        vals = is_validate if isinstance(is_validate, list) else [is_validate] * len(ids)
        out = []
        for rid, val in zip(ids, vals):
            inv, rn = self._inv(val), self._rn(val)
            res = []
            for v in model_versions:
                if rid in self._abort_request_ids:
                    raise AssertionError(f"request {rid} is aborted")
                if not val and v <= self.max_aborted_version:
                    res.append(False)
                    continue
                info = EntryInfo(INVALID_ROLLOUT_INSTANCE_ID, rid // rn, rid % rn, v, 1, val)
                if without_new_reserve_entry:
                    res.append(inv.can_reserve_data_without_new_reserve_entry(info, v))
                else:
                    res.append(inv.can_reserve_data(info, v))
            out.append(res)
        return out[0] if single else out

    @state_locked
    def get_reserve_indicator(self, request_id: int, model_versions: list[int], is_validate: bool = False) -> list[float]:
        """-inf: joins an existing group reservation; -b: needs a new slot, best
        pending buffer is b; +inf: cannot be reserved at that version."""
        inv, rn = self._inv(is_validate), self._rn(is_validate)
        out = []
        for v in model_versions:
            if not is_validate and v <= self.max_aborted_version:
                out.append(float("inf"))
                continue
            info = EntryInfo(INVALID_ROLLOUT_INSTANCE_ID, request_id // rn, request_id % rn, v, 1, is_validate)
            if inv.can_reserve_data_without_new_reserve_entry(info, v):
                out.append(float("-inf"))
            elif inv.can_reserve_data(info, v):
                b = inv.get_max_pending_buffer_id(v + self.staleness) if not is_validate else 0
                out.append(-float(b if b is not None else 0))
            else:
                out.append(float("inf"))
        return out

    @state_locked
    def reserve_rollout_instance_requests(self, rollout_instance_ids, request_ids, model_versions,
                                          guarantee_not_aborted: bool = True, is_validate: bool = False):
        ids = request_ids if isinstance(request_ids, list) else [request_ids]
        n = len(ids)
        insts = rollout_instance_ids if isinstance(rollout_instance_ids, list) else [rollout_instance_ids] * n
        vers = model_versions if isinstance(model_versions, list) else [model_versions] * n
        inv, rn = self._inv(is_validate), self._rn(is_validate)
        bids, eids = [], []
        for inst, rid, v in zip(insts, ids, vers):
            if inst != INVALID_ROLLOUT_INSTANCE_ID and inst not in self.rollout_instance_tracker:
                raise AssertionError(f"rollout instance {inst} is not registered")
            if rid in self._abort_request_ids:
                if guarantee_not_aborted:
                    raise AssertionError(f"request {rid} is aborted")
                self._check_aborted_request(rid, remove=True)
                bids.append(None)
                eids.append(None)
                continue
            if not is_validate and v <= self.max_aborted_version:
                raise AssertionError(f"version {v} <= max aborted version {self.max_aborted_version}")
            info = EntryInfo(inst, rid // rn, rid % rn, v, 1, is_validate)
            b, e = inv.reserve_data(info, None if is_validate else v + self.staleness)
            if b is None:
                raise RuntimeError(f"cannot reserve request {rid} at version {v}: inventory full")
            bids.append(b)
            eids.append(e)
        return bids, eids

    @state_locked
    def update_request_version_tag(self, request_id: int, new_version_tag: int, is_validate: bool = False) -> None:
        self._inv(is_validate).update_request_version_tag(request_id, new_version_tag)
        self.update_request_version(request_id, new_version_tag)

    @state_locked
    def update_request_instance_id(self, request_id: int, new_instance_id, is_validate: bool = False) -> None:
        self._inv(is_validate).update_request_instance_id(request_id, new_instance_id)
        self.update_request_instance(request_id, new_instance_id)

    # -------------------------------------------------------------- abort
    @state_locked
    def check_aborted_model_versions(self, model_versions):
        if isinstance(model_versions, list):
            return [v <= self.max_aborted_version for v in model_versions]
        return model_versions <= self.max_aborted_version

    @state_locked
    def check_aborted_requests(self, request_ids, remove: bool = False):
        if isinstance(request_ids, list):
            return [self._check_aborted_request(r, remove) for r in request_ids]
        return self._check_aborted_request(request_ids, remove)

    @state_locked
    def abort_requests(self, request_ids, abort_group: bool = True, blocking: bool = False) -> set[int]:
        """Abort requests; drop the whole group when fewer than ``alg_rollout_n``
        members would remain."""
        ids = set(request_ids if isinstance(request_ids, list) else [request_ids])
        inv = self.staleness_inventory
        per_prompt: dict[int, list[int]] = {}
        for rid in ids:
            per_prompt.setdefault(rid // self.rollout_n, []).append(rid % self.rollout_n)
        clear: list[int] = []
        for pid, idxs in per_prompt.items():
            if pid not in inv.data_tracker:
                continue
            info = inv.entry_info_of(pid)
            rest = set(info.request_idx) - set(idxs)
            if abort_group and len(rest) < self.alg_rollout_n:
                ids |= {pid * self.rollout_n + r for r in rest}
                clear.append(pid)
            else:
                info.drop_members(idxs)
        # Only reservations are released here; occupied groups stay (they are complete).
        reserved = [p for p in clear
                    if inv.buffers[inv.data_tracker[p][0]].entries[inv.data_tracker[p][1]].category
                    is EntryCategory.RESERVED]
        inv.clear_reserved_entries(reserved)
        self._abort_requests(sorted(ids), blocking)
        return ids

    @state_locked
    def abort_reserved_requests(self, buffer_id: int) -> tuple[int, list[int]]:
        buf = self.staleness_inventory.buffers[buffer_id]
        rids: list[int] = []
        eids = buf.get_reserved_entry_ids()
        for e in eids:
            pid = buf.entries[e].entry_info.prompt_id
            rids.extend(pid * self.rollout_n + i for i in range(self.rollout_n))
        self.abort_requests(rids)
        return len(eids), rids

    def _abort_after_buffer_ready(self, buffer_id: int) -> set[int]:
        """Once every buffer a version may still land in is READY, abort what is
        still in flight at that version (it can no longer be placed)."""
        inv = self.staleness_inventory
        ps_v = self.model_store.version_tag
        ready = inv.ready_buffer_ids()
        if buffer_id >= self.staleness:
            self.check_abort_versions.add(buffer_id - self.staleness)
        versions: list[int] = []
        while self.check_abort_versions:
            v = min(self.check_abort_versions)
            need = set(range(max(v, ps_v), v + self.staleness + 1))
            if not need <= ready:
                break
            versions.append(v)
            self.check_abort_versions.discard(v)
        aborted: set[int] = set()
        for v in versions:
            self.max_aborted_version = max(self.max_aborted_version, v)
            aborted |= self.get_requests_of_abort_version(v)
        if aborted:
            aborted = self.abort_requests(sorted(aborted))
        for b in sorted(ready):
            if b in inv.buffers and inv.buffers[b].get_reserve_entry_num() == 0:
                if ps_v > b:
                    inv.delete_buffer(b)
                else:
                    inv.mark_buffer_for_deletion(b)
        return aborted

    @state_locked
    def handle_ready_buffer(self, buffer_id: int) -> set[int]:
        for cb in self.on_buffer_ready:
            cb(buffer_id)
        return self._abort_after_buffer_ready(buffer_id)

    # ------------------------------------------------------------- occupy
    @state_locked
    def occupy_rollout_instance_request(self, prompt_id: int, request_ids=None, is_validate: bool = False):
        """Commit a finished prompt group.  Returns ``(buffer_id, occupied_count,
        entry_info)`` or ``(None, None, None)`` if every member was aborted."""
        ids = [prompt_id] if request_ids is None else list(request_ids)
        aborted = [self._check_aborted_request(r, remove=True) for r in ids]
        live = [r for r, a in zip(ids, aborted) if not a]
        inv = self._inv(is_validate)
        for r in live:
            if r in self._status:
                self.remove_request(r)
        if not live:
            if prompt_id in inv.data_tracker:
                raise AssertionError(f"prompt {prompt_id} fully aborted but still in the inventory")
            return None, None, None
        bid, eid, occ = inv.occupy_data_with_reserve(prompt_id)
        return bid, occ, inv.buffers[bid].entries[eid].entry_info

    @state_locked
    def get_buffer_status(self, buffer_id: int, is_validate: bool = False) -> BufferStatus | None:
        inv = self._inv(is_validate)
        return inv.get_buffer_status(buffer_id) if buffer_id in inv.buffers else None

    @state_locked
    def ensure_train_buffer_exists(self, buffer_id: int) -> None:
        self.staleness_inventory.ensure_buffer_exists(buffer_id)

    @state_locked
    def consume_buffer(self, buffer_id: int, is_validate: bool = False) -> list[EntryInfo]:
        """Entries of a READY buffer's training region, in slot order."""
        inv = self._inv(is_validate)
        buf = inv.buffers[buffer_id]
        if buf.get_status() not in (BufferStatus.READY, BufferStatus.READY_WITH_CAPACITY):
            raise RuntimeError(f"buffer {buffer_id} is not ready ({buf.get_status()})")
        return [e.entry_info for e in buf.entries[: buf.ready_num_entries]]

    @state_locked
    def get_min_pending_buffer(self, is_validate: bool = False) -> int:
        inv = self._inv(is_validate)
        p = inv.get_buffers_with_capacity()
        return min(p) if p else inv.buffer_id

    def maybe_delete_buffer(self, buffer_id: int, is_validate: bool = False) -> None:
        inv = self._inv(is_validate)
        if is_validate:
            inv.delete_buffer(buffer_id)
            return
        marked = inv.get_ready_for_delete_buffer_ids()
        if buffer_id in marked:
            for b in sorted(marked):
                if b <= buffer_id:
                    inv.delete_buffer(b)

    # --------------------------------------------------- push / pull lock
    def acquire_exclusive_push(self, timeout: float | None = None) -> bool:
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._rw:
            while self._exclusive_push_locked or self._shared_pull_count > 0:
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._rw.wait(left)
            self._exclusive_push_locked = True
            return True

    def release_exclusive_push(self) -> None:
        with self._rw:
            self._exclusive_push_locked = False
            self._rw.notify_all()

    def acquire_shared_pull(self, timeout: float | None = None) -> bool:
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._rw:
            while self._exclusive_push_locked:
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._rw.wait(left)
            self._shared_pull_count += 1
            return True

    def release_shared_pull(self) -> None:
        with self._rw:
            self._shared_pull_count -= 1
            if self._shared_pull_count < 0:
                raise RuntimeError("shared pull released more often than acquired")
            self._rw.notify_all()

    def lock_state(self) -> tuple[bool, int]:
        with self._rw:
            return self._exclusive_push_locked, self._shared_pull_count

    # ---------------------------------------------------------- push/pull
    def push_model(self, version: int, state: Any = None) -> None:
        """Publish ``version`` (the caller holds the exclusive push lock while it
        writes the weights).  Deletes consumed buffers and notifies listeners."""
        with self._state_lock:
            if version < self.model_store.version_tag:
                raise ValueError(f"version {version} < published {self.model_store.version_tag}")
            self.model_store.version_tag = int(version)
            if state is not None:
                self.model_store.state = state
            self.model_store.push_time = time.time()
            self.maybe_delete_buffer(version - 1)
            self._refresh_running_min_version()
        for cb in self.on_version_published:
            cb(int(version))

    def pull_model(self, instance_id=None) -> tuple[int, Any]:
        """Current ``(version, state)``; records the instance's new version."""
        with self._state_lock:
            v, s = self.model_store.version_tag, self.model_store.state
            if instance_id is not None:
                self.set_rollout_instance_model_version(instance_id, v)
            return v, s

    # -------------------------------------------------------- diagnostics
    @state_locked
    def snapshot(self) -> dict:
        inv = self.staleness_inventory
        return {
            "ps_version": self.model_store.version_tag,
            "max_aborted_version": self.max_aborted_version,
            "buffers": {b: inv.buffers[b].get_status().name for b in sorted(inv.buffers)},
            "occupied": {b: inv.buffers[b].count(EntryCategory.OCCUPIED) for b in sorted(inv.buffers)},
            "reserved": {b: inv.buffers[b].count(EntryCategory.RESERVED) for b in sorted(inv.buffers)},
            "requests": {s.name: len(v) for s, v in self._by_status.items() if v},
        }


__all__ = ["ModelStore", "PSManager", "RolloutInstanceStatus", "RequestStatus"]
