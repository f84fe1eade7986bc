"""Lock helpers (C35): busy-polling method lock, exclusive-push / shared-pull
context managers over the PS reader-writer lock, and a version waiter.

Reference: ``psrl/utils/ray/lock_context.py:44-248``.
"""

from __future__ import annotations

import contextlib
import functools
import threading
import time


def add_busy_polling_lock(cls):
    """Class decorator: methods named in ``cls.__locked_methods__`` (or all public
    methods if absent) run under one re-entrant lock per instance."""
    names = getattr(cls, "__locked_methods__", None)
    orig_init = cls.__init__

    def __init__(self, *a, **k):
        self._busy_lock = threading.RLock()
        orig_init(self, *a, **k)

    cls.__init__ = __init__
    for name, fn in list(vars(cls).items()):
        if name.startswith("_") or not callable(fn) or (names is not None and name not in names):
            continue

        def make(f):
            @functools.wraps(f)
            def locked(self, *a, **k):
                with self._busy_lock:
                    return f(self, *a, **k)
            return locked
        setattr(cls, name, make(fn))
    return cls


@contextlib.contextmanager
def exclusive_push_model_context(ps, timeout: float | None = 600.0, poll_s: float = 0.0):
    if not ps.acquire_exclusive_push(timeout):
        raise TimeoutError("exclusive push lock not acquired")
    try:
        yield
    finally:
        ps.release_exclusive_push()


@contextlib.contextmanager
def shared_pull_model_context(ps, timeout: float | None = 600.0):
    if not ps.acquire_shared_pull(timeout):
        raise TimeoutError("shared pull lock not acquired")
    try:
        yield
    finally:
        ps.release_shared_pull()


def wait_for_version(get_version, target: int, timeout: float = 600.0, poll_s: float = 0.01) -> int:
    """Poll ``get_version()`` until it reaches ``target`` (the reference's version waiter)."""
    t0 = time.monotonic()
    while True:
        v = get_version()
        if v >= target:
            return v
        if time.monotonic() - t0 > timeout:
            raise TimeoutError(f"version {target} not reached (at {v})")
        time.sleep(poll_s)


class RWLock:
    """Process-local reader-writer lock with bounded waits: the optimizer step of
    a colocated trainer holds it exclusively (in-place parameter update) while
    the rollout engine's weight pull holds it shared (reads the parameters)."""

    def __init__(self):
        self._cv = threading.Condition()
        self._writer = False
        self._readers = 0

    def acquire_exclusive(self, timeout: float | None = None) -> bool:
        with self._cv:
            return self._cv.wait_for(lambda: not self._writer and self._readers == 0, timeout) and \
                self._set_writer()

    def _set_writer(self) -> bool:
        self._writer = True
        return True

    def release_exclusive(self) -> None:
        with self._cv:
            self._writer = False
            self._cv.notify_all()

    def acquire_shared(self, timeout: float | None = None) -> bool:
        with self._cv:
            if not self._cv.wait_for(lambda: not self._writer, timeout):
                return False
            self._readers += 1
            return True

    def release_shared(self) -> None:
        with self._cv:
            if self._readers <= 0:
                raise RuntimeError("shared lock released more often than acquired")
            self._readers -= 1
            self._cv.notify_all()

    @contextlib.contextmanager
    def exclusive(self, timeout: float | None = 600.0):
        if not self.acquire_exclusive(timeout):
            raise TimeoutError("exclusive lock not acquired")
        try:
            yield
        finally:
            self.release_exclusive()

    @contextlib.contextmanager
    def shared(self, timeout: float | None = 600.0):
        if not self.acquire_shared(timeout):
            raise TimeoutError("shared lock not acquired")
        try:
            yield
        finally:
            self.release_shared()
