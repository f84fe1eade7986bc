"""GPU: VMM sleep/wake regions, KV block copies (device <-> pinned host)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_vmm_sleep_wake_backup_and_release():
    from psrl_b200.parallel.memory import MemoryPool
    pool = MemoryPool("cuda:0")
    t = pool.tensor("weights", (1 << 24,), torch.bfloat16)       # 32 MB
    kv = pool.tensor("kv", (1 << 26,), torch.float32)            # 256 MB
    t.copy_(torch.arange(t.numel(), device="cuda").bfloat16())
    kv.fill_(3.0)
    ref = t.clone()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    pool.sleep("kv", backup=False)
    pool.sleep("weights", backup=True)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 - free0 >= (1 << 28)                             # physical memory returned
    assert not pool.is_awake("kv")
    pool.wake("weights")
    pool.wake("kv")
    assert torch.equal(t, ref)                                   # restored from the host copy
    assert float(kv.abs().sum()) == 0.0                          # fresh pages are zero-filled


def test_kv_copy_blocks_device_host_roundtrip():
    from psrl_b200.rollout.kv_offload import copy_blocks
    L, nb, nkv, bs, d = 3, 10, 2, 16, 128
    k = [torch.randn(nb, nkv, bs, d, device="cuda").bfloat16() for _ in range(L)]
    v = [torch.randn(nb, nkv, bs, d, device="cuda").bfloat16() for _ in range(L)]
    hk = [torch.zeros(4, nkv, bs, d, dtype=torch.bfloat16, pin_memory=True) for _ in range(L)]
    hv = [torch.zeros(4, nkv, bs, d, dtype=torch.bfloat16, pin_memory=True) for _ in range(L)]
    copy_blocks(k, v, hk, hv, [7, 2, 5], [0, 1, 3], torch.device("cuda"))
    torch.cuda.synchronize()
    for l in range(L):
        assert torch.equal(hk[l][0], k[l][7].cpu()) and torch.equal(hv[l][3], v[l][5].cpu())
    k2 = [torch.zeros_like(x) for x in k]
    v2 = [torch.zeros_like(x) for x in v]
    copy_blocks(hk, hv, k2, v2, [0, 1, 3], [4, 8, 9], torch.device("cuda"))
    torch.cuda.synchronize()
    for l in range(L):
        assert torch.equal(k2[l][4], k[l][7]) and torch.equal(v2[l][9], v[l][5])
