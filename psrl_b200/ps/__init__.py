"""Parameter Server: staleness inventory, request tracking and the PS manager."""

from .manager import ModelStore, PSManager, RolloutInstanceStatus
from .request_tracker import PSRL_RequestStatus, RequestStatus, RequestStatusTracker
from .staleness import (
    INVALID_ROLLOUT_INSTANCE_ID,
    BufferStatus,
    Entry,
    EntryCategory,
    EntryInfo,
    InventoryError,
    StalenessBuffer,
    StalenessInventory,
)

__all__ = [
    "BufferStatus",
    "Entry",
    "EntryCategory",
    "EntryInfo",
    "INVALID_ROLLOUT_INSTANCE_ID",
    "InventoryError",
    "ModelStore",
    "PSManager",
    "PSRL_RequestStatus",
    "RequestStatus",
    "RequestStatusTracker",
    "RolloutInstanceStatus",
    "StalenessBuffer",
    "StalenessInventory",
]
