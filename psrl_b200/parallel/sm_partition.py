"""SM partitioning between a trainer and a rollout engine on one GPU.

Training GEMMs from cuBLAS are persistent kernels that hold every SM until they
finish, so decode kernels queued behind them wait even on a high-priority
stream.  :func:`trainer_stream` returns a stream of a CUDA green context that
owns all SMs except ``reserve_sms`` (rounded up to the split granularity): the
trainer launches on it, the rollout engine keeps an ordinary stream, so decode
kernels always find the reserved SMs free and use the whole GPU while the
trainer is idle.  Implemented in ``csrc/green.cpp``.
"""

from __future__ import annotations

import torch

from ..ops._ext import ext


def trainer_stream(device: torch.device, reserve_sms: int, priority: int = 0):
    """(stream, info) — ``info`` has ``sms`` (trainer SMs), ``reserved_sms`` and
    ``total_sms``."""
    dev = torch.device(device)
    info = dict(ext().green_partition(int(dev.index or 0), int(reserve_sms), int(priority)))
    return torch.cuda.ExternalStream(int(info["stream"]), device=dev), info
