"""Debug-build kernel bounds checks (``csrc/checks.cuh``).

Build with ``PSRL_KERNEL_CHECKS=1 python setup.py build_ext --inplace`` and
the kernels that index memory through caller-supplied tables (paged-KV block
tables and lengths, copy segments, optimizer shard offsets, KV block moves)
range-check every such index.  A failed check skips the access and leaves a
record on the device; :func:`check_kernel_bounds` reads it and raises.  In a
regular build both functions are free and report nothing.
"""

from __future__ import annotations

from ._ext import ext

CODES = {
    61: "paged prefill: kv_len above max_blocks * block_size",
    62: "paged prefill: block id out of range",
    63: "decode attention: kv_len above max_blocks * block_size",
    64: "decode attention: block id out of range",
    65: "peer copy (copy_segments / scatter_segments / copy_rows): destination offset out of range",
    66: "peer optimizer: shard offset out of range",
    67: "kv_copy_blocks: block id out of range",
}


def kernel_checks_enabled() -> bool:
    return bool(ext().kernel_checks_enabled())


def kernel_check_record(clear: bool = True) -> list[int]:
    """[code, a, b, value, bound, failures] of the first failed check on the
    current device since the last clear (zeros if none).  Synchronises."""
    return [int(v) for v in ext().kernel_check_status(bool(clear))]


def check_kernel_bounds(clear: bool = True) -> None:
    rec = kernel_check_record(clear)
    if rec[0]:
        raise RuntimeError(f"kernel bounds check {rec[0]} ({CODES.get(rec[0], 'unknown')}): context "
                           f"({rec[1]}, {rec[2]}), value {rec[3]}, bound {rec[4]}; {rec[5]} failed checks")
