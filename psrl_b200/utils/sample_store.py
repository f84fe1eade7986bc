"""Keyed sample-field store (C28 / N12): the TransferQueue role.

Trajectory fields are addressed by uid keys inside a partition ("train" /
"val"); ``KVBatchMeta`` names a batch of keys with tags.  The store lives in
the driver process (remote producers reach it over RPC), so payloads move
once and device tensors stay on their device when producer and consumer share
a process.  API: ``kv_batch_put / kv_batch_get / kv_clear / kv_list``.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, field


@dataclass
class KVBatchMeta:
    keys: list
    tags: list = field(default_factory=list)
    partition: str = "train"


class SampleStore:
    def __init__(self):
        self._data: dict[str, dict] = {"train": {}, "val": {}}
        self._lock = threading.Lock()

    def kv_batch_put(self, keys, fields: list[dict], partition: str = "train", tags=None) -> KVBatchMeta:
        if len(keys) != len(fields):
            raise ValueError("keys and fields differ in length")
        with self._lock:
            part = self._data.setdefault(partition, {})
            for k, f in zip(keys, fields):
                part.setdefault(str(k), {}).update(f)
        return KVBatchMeta([str(k) for k in keys], list(tags or []), partition)

    def kv_batch_get(self, meta: KVBatchMeta, select: list[str] | None = None) -> list[dict]:
        with self._lock:
            part = self._data.get(meta.partition, {})
            out = []
            for k in meta.keys:
                rec = part[str(k)]
                out.append({f: rec[f] for f in select} if select else dict(rec))
            return out

    def kv_clear(self, keys, partition: str = "train") -> int:
        with self._lock:
            part = self._data.get(partition, {})
            n = 0
            for k in keys:
                if part.pop(str(k), None) is not None:
                    n += 1
            return n

    def kv_list(self, partition: str = "train") -> list[str]:
        with self._lock:
            return list(self._data.get(partition, {}))

    def __len__(self) -> int:
        with self._lock:
            return sum(len(p) for p in self._data.values())
