"""Loader for the host-only native modules (no CUDA).

``router()`` returns the compiled router core (``csrc_host/router_core.cpp``):
the in-tree build from ``python setup.py build_ext --inplace`` when present,
otherwise a one-time compile of the same source with the C++ toolchain into
``build/native`` under the repository, so a fresh checkout works without the
CUDA build.
"""

from __future__ import annotations

import os
import threading

_lock = threading.Lock()
_router_mod = None


def router():
    global _router_mod
    if _router_mod is not None:
        return _router_mod
    with _lock:
        if _router_mod is None:
            try:
                from . import _router as mod
            except ImportError:
                from torch.utils.cpp_extension import load
                here = os.path.dirname(os.path.abspath(__file__))
                bdir = os.path.join(os.path.dirname(here), "build", "native")
                os.makedirs(bdir, exist_ok=True)
                mod = load(name="_router", sources=[os.path.join(here, "csrc_host", "router_core.cpp")],
                           extra_cflags=["-O3", "-std=c++17"], build_directory=bdir, verbose=False)
            _router_mod = mod
    return _router_mod
