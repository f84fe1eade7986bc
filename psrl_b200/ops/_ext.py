"""Loader for the compiled sm_100a kernel library (``psrl_b200/_C*.so``).

On a machine with a CUDA device the extension is mandatory: any CUDA tensor
reaching an op without the library loaded raises instead of silently running a
PyTorch fallback.  CPU tensors use the PyTorch reference implementations.
"""

from __future__ import annotations

import importlib

_EXT = None
_ERR: Exception | None = None

# Kernel launches issued through this module (host-side count).  CUDA-graph
# replays are added by the engine from the count recorded at capture time.
LAUNCHES = 0
_KERNELS_PER_CALL = {"rmsnorm_bwd": 1, "sqnorm_accumulate_": 2, "attn_varlen_bwd": 2}


class _Counted:
    """Proxy over the extension module that counts kernel launches."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        per = _KERNELS_PER_CALL.get(name, 1)

        def wrapped(*a, **k):
            global LAUNCHES
            n = per
            if name == "attn_decode" and len(a) > 6 and int(a[6]) > 1:
                n = 2
            LAUNCHES += n
            return fn(*a, **k)

        return wrapped


def launches() -> int:
    return LAUNCHES


def add_launches(n: int) -> None:
    global LAUNCHES
    LAUNCHES += int(n)


def ext():
    """Return the ``psrl_b200._C`` module or raise with the build command."""
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            _EXT = _Counted(importlib.import_module("psrl_b200._C"))
        except Exception as exc:  # pragma: no cover - depends on the build
            _ERR = exc
    if _EXT is None:
        raise RuntimeError(
            "psrl_b200 CUDA kernels are not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_ERR})"
        )
    return _EXT


def has_ext() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False
