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
