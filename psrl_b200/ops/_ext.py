"""Loader for the compiled sm_100a kernel library (``psrl_b200/_C*.so``).

On a machine with a CUDA device the extension is mandatory: any CUDA tensor
reaching an op without the library loaded raises instead of silently running a
PyTorch fallback.  CPU tensors use the PyTorch reference implementations.
"""

from __future__ import annotations

import importlib

_EXT = None
_ERR: Exception | None = None


def ext():
    """Return the ``psrl_b200._C`` module or raise with the build command."""
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            _EXT = importlib.import_module("psrl_b200._C")
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
