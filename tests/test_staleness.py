"""Staleness inventory: Reserve / Occupy / Consume semantics and invariants.

Scenarios mirror the reference's ``tests/staleness/test_staleness_controller.py``
(READY/STUCK/PENDING transitions, reserve window, scalar/list request_idx) and
add a property-based protocol simulation that checks the staleness bound after
every mutation.
"""

import random

import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from psrl_b200.ps.staleness import (
    BufferStatus,
    EntryCategory,
    EntryInfo,
    InventoryError,
    StalenessBuffer,
    StalenessInventory,
)

INST = (0, 0)


def info(pid, idx=0, ver=0):
    return EntryInfo(INST, pid, idx, ver)


def test_entry_info_normalises_members():
    e = EntryInfo(INST, 3, [0, 1], [2, 1])
    assert e.get_entry_version() == 1
    assert e.get_all_request_ids(4) == [12, 13]
    assert e.rollout_instance_id == [INST, INST]
    s = EntryInfo(INST, 3, 2, 5)
    assert s.request_idx == [2] and s.model_version == [5]
    assert s.add_member(1, 4, (1, 0)) is True
    assert s.add_member(1, 4, (1, 0)) is False
    assert s.get_entry_version() == 4
    s.drop_members([2])
    assert s.request_idx == [1] and s.model_version == [4]


def test_buffer_status_transitions():
    b = StalenessBuffer(4, 4, 1)
    assert b.get_status() is BufferStatus.PENDING
    for i in range(4):
        b.insert(i, EntryCategory.RESERVED, info(i))
    assert b.get_status() is BufferStatus.STUCK
    for i in range(4):
        b.insert(i, EntryCategory.OCCUPIED, info(i))
    assert b.get_status() is BufferStatus.READY
    r = StalenessBuffer(6, 4, 1)
    for i in range(4):
        r.insert(i, EntryCategory.OCCUPIED, info(i))
    assert r.get_status() is BufferStatus.READY_WITH_CAPACITY


def test_reserve_takes_highest_buffer_last_slot():
    inv = StalenessInventory(4, 4, staleness=2, rollout_n=1)
    b, e = inv.reserve_data(info(0, ver=0), max_staleness_buffer_id=2)
    assert (b, e) == (2, 3)
    assert set(inv.buffers) == {0, 1, 2}
    b, e = inv.reserve_data(info(1, ver=0), 2)
    assert (b, e) == (2, 2)
    inv.check_invariants()


def test_reserve_is_idempotent_for_group_members():
    inv = StalenessInventory(4, 4, staleness=1, rollout_n=4)
    loc = inv.reserve_data(EntryInfo(INST, 7, 0, 0), 1)
    assert inv.reserve_data(EntryInfo((1, 0), 7, 1, 1), 1) == loc
    assert inv.reserve_data(EntryInfo((1, 0), 7, 1, 1), 1) == loc
    e = inv.entry_info_of(7)
    assert e.request_idx == [0, 1] and e.model_version == [0, 1]
    assert e.get_entry_version() == 0


def test_occupy_is_greedy_lowest_buffer():
    inv = StalenessInventory(2, 2, staleness=1, rollout_n=1)
    inv.reserve_data(info(0, ver=0), 1)      # reserved in buffer 1
    b, e, n = inv.occupy_data_with_reserve(0)
    assert (b, e, n) == (0, 0, 1)            # lands in buffer 0
    assert inv.buffers[1].get_status() is BufferStatus.PENDING
    inv.check_invariants()


def test_reservation_exchange_keeps_occupied_prefix():
    inv = StalenessInventory(2, 2, staleness=0, rollout_n=1)
    inv.reserve_data(info(0), 0)   # (0,1)
    inv.reserve_data(info(1), 0)   # (0,0)
    assert inv.buffers[0].get_status() is BufferStatus.STUCK
    # prompt 0 (slot 1) finishes first: prompt 1's reservation moves to slot 1
    b, e, n = inv.occupy_data_with_reserve(0)
    assert (b, e) == (0, 0)
    assert inv.data_tracker[1] == (0, 1)
    inv.check_invariants()
    inv.occupy_data_with_reserve(1)
    assert inv.buffers[0].get_status() is BufferStatus.READY


def test_cannot_reserve_outside_window():
    inv = StalenessInventory(1, 1, staleness=1, rollout_n=1)
    inv.reserve_data(info(0, ver=0), 1)      # buffer 1 full
    inv.reserve_data(info(1, ver=0), 1)      # buffer 0
    assert inv.can_reserve_data(info(2, ver=0), 0) is False
    assert inv.reserve_data(info(2, ver=0), 1) == (None, None)
    assert inv.can_reserve_data(info(2, ver=1), 1) is True


def test_clear_occupied_compacts():
    inv = StalenessInventory(3, 3, staleness=0, rollout_n=1)
    for p in range(3):
        inv.reserve_data(info(p), 0)
    for p in range(3):
        inv.occupy_data_with_reserve(p)
    inv.clear_occupied_entries(0)
    assert inv.buffers[0].get_first_non_occupied() == 2
    inv.check_invariants()


def test_validation_inventory_has_no_staleness():
    inv = StalenessInventory(8, 4, staleness=3, rollout_n=1, is_validate=True)
    assert inv.staleness is None and inv.num_entries == 4
    b, e = inv.reserve_data(info(0, ver=9), None)
    assert b == 0
    inv.occupy_data_with_reserve(0)
    inv.check_invariants()


def test_redundant_rollout_spare_slots():
    # 3 slots, 2 make a batch: the first reservation takes the spare slot 2.
    inv = StalenessInventory(3, 2, staleness=0, rollout_n=1)
    locs = [inv.reserve_data(info(p), 0) for p in range(3)]
    assert locs[0] == (0, 2)
    for p in (1, 2, 0):
        inv.occupy_data_with_reserve(p)
        inv.check_invariants()
    assert inv.buffers[0].get_status() in (BufferStatus.READY, BufferStatus.READY_WITH_CAPACITY)


def test_mark_and_delete_buffer():
    inv = StalenessInventory(1, 1, staleness=0, rollout_n=1)
    inv.reserve_data(info(0), 0)
    with pytest.raises(InventoryError):
        inv.mark_buffer_for_deletion(0)
    inv.occupy_data_with_reserve(0)
    inv.mark_buffer_for_deletion(0)
    assert inv.get_ready_for_delete_buffer_ids() == {0}
    inv.delete_buffer(0)
    assert 0 not in inv.buffers and 0 not in inv.data_tracker


def _simulate(seed: int, staleness: int, entries: int, ready: int, steps: int):
    """Drive the inventory like the async runtime does and check invariants.

    Model versions advance when the lowest buffer is READY (the trainer
    consumes it).  Requests reserve at dispatch with the current version and
    occupy later in random order.
    """
    rng = random.Random(seed)
    inv = StalenessInventory(entries, ready, staleness, rollout_n=1)
    version = 0
    next_pid = 0
    inflight: list[tuple[int, int]] = []   # (pid, version)
    consumed = 0
    for _ in range(steps):
        op = rng.random()
        if op < 0.5:
            e = info(next_pid, ver=version)
            if inv.can_reserve_data(e, version):
                b, _ = inv.reserve_data(e, version + staleness)
                if b is not None:
                    assert version <= b <= version + staleness
                    inflight.append((next_pid, version))
                    next_pid += 1
        elif inflight:
            pid, v = inflight.pop(rng.randrange(len(inflight)))
            if pid in inv.data_tracker:
                b, e, _ = inv.occupy_data_with_reserve(pid)
                assert v <= b <= v + staleness, (v, b)
        inv.check_invariants()
        # trainer consumes buffer `version` once ready
        if version in inv.buffers and inv.get_buffer_status(version) in (
                BufferStatus.READY, BufferStatus.READY_WITH_CAPACITY):
            for ent in inv.buffers[version].entries[:ready]:
                assert ent.category is EntryCategory.OCCUPIED
                assert ent.entry_info.get_entry_version() >= version - staleness
            if inv.buffers[version].get_reserve_entry_num() == 0:
                inv.delete_buffer(version)
            else:
                inv.mark_buffer_for_deletion(version)
            version += 1
            consumed += 1
            inv.check_invariants()
    return consumed


@pytest.mark.parametrize("staleness", [0, 1, 3])
def test_protocol_simulation_progresses(staleness):
    consumed = _simulate(seed=staleness, staleness=staleness, entries=4, ready=4, steps=600)
    assert consumed > 10


@settings(max_examples=60, deadline=None, derandomize=True)
@given(seed=st.integers(0, 10_000), staleness=st.integers(0, 4), ready=st.integers(1, 6),
       extra=st.integers(0, 2))
def test_protocol_simulation_property(seed, staleness, ready, extra):
    _simulate(seed, staleness, ready + extra, ready, steps=250)


def test_reservation_exchange_with_parked_spare_entry():
    """Regression: a wasted redundant rollout parked in a spare slot sits behind
    the EMPTY slots; reservations and reservation exchanges must take the last
    EMPTY slot, not the parked entry."""
    assert _simulate(477, 3, 3, 1, steps=250) > 0
