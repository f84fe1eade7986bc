"""tcgen05/TMEM GEMM entry points (``csrc/gemm_sm100.cu``).

* :func:`tc_linear` — ``x @ w.T`` (bf16, K-major operands, K % 64 == 0).
* :func:`tc_linear_logprob` — LM-head log-probabilities/entropy with the
  log-sum-exp fused into the GEMM epilogue (no [T, V] logits in memory).

Each call passes a device error flag; a nonzero value means a bounded wait
inside the kernel gave up (the kernel then freed its tensor memory and
returned) and is raised here.
"""

from __future__ import annotations

import torch

from ._ext import ext

_ERR: dict = {}


def _err(device) -> torch.Tensor:
    e = _ERR.get(device)
    if e is None:
        # [code, block x, block y, block z, warp, iteration, -, -] of the first failure
        e = torch.zeros(8, dtype=torch.int32, device=device)
        _ERR[device] = e
    return e


def check_errors(device=None) -> None:
    for dev, e in _ERR.items():
        if device is not None and dev != device:
            continue
        rec = e.tolist()
        if rec[0]:
            e.zero_()
            if rec[0] == 51:
                raise RuntimeError(f"cross-GPU flag barrier timed out: rank {rec[1]} last published epoch "
                                   f"{rec[2]}, this rank waited for {rec[3]}")
            raise RuntimeError(f"tcgen05 kernel reported error code {rec[0]} (a bounded wait expired; "
                               f"block ({rec[1]}, {rec[2]}, {rec[3]}), warp {rec[4]}, iteration {rec[5]})")


def supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
            and x.shape[1] % 64 == 0 and x.stride(1) == 1 and w.stride(1) == 1 and w.shape[0] % 8 == 0)


def tc_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return ext().tc_gemm(x, w, _err(x.device))


def tc_linear_logprob(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, temperature: float = 1.0):
    lp, ent, lse = ext().tc_linear_logprob(h.contiguous(), w, labels.long(), float(temperature), _err(h.device))
    return lp, ent, lse
