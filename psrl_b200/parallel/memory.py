"""GPU memory pause/resume for colocated roles (C31 / N9 / N10).

A ``MemoryPool`` hands out tensors that live in driver virtual-memory regions
(``VmmRegion``, ``csrc/vmm.cpp``).  ``sleep(tag)`` releases the physical memory
of every region with that tag (optionally keeping a pinned host copy) while
the tensors keep their addresses — so CUDA graphs captured on them stay valid
— and ``wake(tag)`` maps new memory at the same addresses and restores the
copy.  Used to time-share GPUs between the trainer and the rollout engine (the
reference does this with torch_memory_saver).  Tensors must not be touched
while their region sleeps.
"""

from __future__ import annotations

import torch

from ..ops import ext

_TYPESTR = {torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4", torch.int64: "<i8",
            torch.uint8: "|u1", torch.int16: "<i2"}


class _CAI:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3}


def wrap_device_memory(ptr: int, shape, dtype, device) -> torch.Tensor:
    """A tensor viewing externally managed device memory (it does not own it)."""
    if dtype == torch.bfloat16:
        return torch.as_tensor(_CAI(ptr, shape, "<i2"), device=device).view(torch.bfloat16)
    return torch.as_tensor(_CAI(ptr, shape, _TYPESTR[dtype]), device=device)


class MemoryPool:
    def __init__(self, device):
        self.device = torch.device(device)
        self.regions: dict[str, list] = {}
        self._keep: list = []

    def tensor(self, tag: str, shape, dtype=torch.bfloat16) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        reg = ext().VmmRegion(int(nbytes), self.device.index or 0)
        self.regions.setdefault(tag, []).append(reg)
        t = wrap_device_memory(reg.ptr(), shape, dtype, self.device)
        self._keep.append(reg)
        return t

    def sleep(self, tag: str, backup: bool = False) -> int:
        freed = 0
        for r in self.regions.get(tag, []):
            if r.awake():
                r.sleep(backup)
                freed += r.size()
        return freed

    def wake(self, tag: str) -> int:
        n = 0
        for r in self.regions.get(tag, []):
            if not r.awake():
                r.wake()
                n += r.size()
        return n

    def is_awake(self, tag: str) -> bool:
        return all(r.awake() for r in self.regions.get(tag, []))
