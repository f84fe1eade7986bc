"""Concurrency limiters (C37): a cross-process slot limiter on ``fcntl`` file
locks and a token bucket (reference ``psrl/utils/concurrency/{slot,token_bucket}.py``)."""

from __future__ import annotations

import contextlib
import fcntl
import os
import threading
import time


class FileSlotLimiter:
    """At most ``n_slots`` holders across processes on one host."""

    def __init__(self, directory: str, n_slots: int, name: str = "slot"):
        self.dir = os.path.expanduser(directory)
        os.makedirs(self.dir, exist_ok=True)
        self.paths = [os.path.join(self.dir, f"{name}.{i}.lock") for i in range(n_slots)]

    @contextlib.contextmanager
    def slot(self, timeout: float = 600.0, poll_s: float = 0.01):
        t0 = time.monotonic()
        while True:
            for p in self.paths:
                fh = open(p, "a+")
                try:
                    fcntl.flock(fh.fileno(), fcntl.LOCK_EX | fcntl.LOCK_NB)
                except BlockingIOError:
                    fh.close()
                    continue
                try:
                    yield p
                finally:
                    fcntl.flock(fh.fileno(), fcntl.LOCK_UN)
                    fh.close()
                return
            if time.monotonic() - t0 > timeout:
                raise TimeoutError("no free slot")
            time.sleep(poll_s)


class TokenBucket:
    def __init__(self, rate_per_s: float, capacity: float):
        self.rate = float(rate_per_s)
        self.capacity = float(capacity)
        self.tokens = float(capacity)
        self.t = time.monotonic()
        self._lock = threading.Lock()

    def _refill(self):
        now = time.monotonic()
        self.tokens = min(self.capacity, self.tokens + (now - self.t) * self.rate)
        self.t = now

    def try_acquire(self, n: float = 1.0) -> bool:
        with self._lock:
            self._refill()
            if self.tokens >= n:
                self.tokens -= n
                return True
            return False

    def acquire(self, n: float = 1.0, timeout: float = 60.0) -> None:
        t0 = time.monotonic()
        while not self.try_acquire(n):
            if time.monotonic() - t0 > timeout:
                raise TimeoutError("token bucket timeout")
            time.sleep(min(0.05, n / max(self.rate, 1e-9)))
