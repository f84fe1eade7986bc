"""GPU test of the allocation-free decode entry point, called through its
exported C symbol with ctypes (the way a C/C++ caller that cannot allocate
device memory would use it), against the regular decode entry point.

Kept in a file that sorts last so a run that stops at the first failure has
already run every other test."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, EBADARG, ETOOBIG = 0, 1, 2
SCRATCH_FLOATS = 16 * 1024 * 1024 // 4


def _entry():
    import psrl_b200._C as C   # loads the library into this process
    lib = ctypes.CDLL(C.__file__)
    fn = lib.psrl_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_void_p]
    return fn


def _case(seed, ctx, nq=16, nkv=2, d=128, bs=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nblk = sum((c + bs - 1) // bs for c in ctx) + 2
    kc = torch.randn(nblk, nkv, bs, d, device="cuda", generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, d, device="cuda", generator=g).bfloat16()
    maxb = max((c + bs - 1) // bs for c in ctx) + 1
    bt = torch.zeros(len(ctx), maxb, dtype=torch.int32)
    perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(seed)).tolist()
    k = 0
    for i, c in enumerate(ctx):
        nb = (c + bs - 1) // bs
        bt[i, :nb] = torch.tensor(perm[k:k + nb])
        k += nb
    q = torch.randn(len(ctx), nq, d, device="cuda", generator=g).bfloat16()
    return q, kc, vc, bt.cuda(), torch.tensor(ctx, dtype=torch.int32, device="cuda")


def _call(fn, q, kc, vc, bt, lens, out, splits):
    B, nq, d = q.shape
    return fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
              B, nq, kc.shape[1], d, kc.shape[2], bt.shape[1], splits, 1.0 / math.sqrt(d),
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("splits", [1, 4])
def test_noalloc_matches_regular_entry_point_twice(splits):
    from psrl_b200.ops import paged_decode_attention
    from psrl_b200.ops.attention import paged_attention_ref
    fn = _entry()
    # two calls in a row with different inputs: the shared scratch must not leak
    for seed, ctx in ((1, [1, 70, 300, 1500, 64]), (2, [900, 5, 128, 2000, 33, 260, 1])):
        q, kc, vc, bt, lens = _case(seed, ctx)
        out = torch.full_like(q, float("nan"))
        assert _call(fn, q, kc, vc, bt, lens, out, splits) == OK
        torch.cuda.synchronize()
        ref = paged_decode_attention(q, kc, vc, bt, lens, splits=splits)
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-2, rtol=2e-2)
        # and directly against the plain fp32 PyTorch attention over the same pages
        B = q.shape[0]
        cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
        oracle = paged_attention_ref(q.float(), kc.float(), vc.float(), cu, lens, bt, 1.0 / math.sqrt(q.shape[-1]))
        torch.testing.assert_close(out.float(), oracle, atol=2e-2, rtol=2e-2)


def test_noalloc_rejects_oversize_and_bad_args():
    fn = _entry()
    q, kc, vc, bt, lens = _case(3, [100, 200])
    out = torch.zeros_like(q)
    B, nq = q.shape[0], q.shape[1]
    too_many = SCRATCH_FLOATS // (B * nq * 129) + 1
    if too_many <= 32:
        assert _call(fn, q, kc, vc, bt, lens, out, too_many) == ETOOBIG
    big_q = torch.zeros(4096, nq, 128, device="cuda", dtype=torch.bfloat16)
    big_bt = torch.zeros(4096, bt.shape[1], device="cuda", dtype=torch.int32)
    big_lens = torch.ones(4096, device="cuda", dtype=torch.int32)
    big_out = torch.zeros_like(big_q)
    assert _call(fn, big_q, kc, vc, big_bt, big_lens, big_out, 8) == ETOOBIG
    assert fn(None, None, None, None, None, None, 1, 16, 2, 128, 64, 1, 1, 1.0, None) == EBADARG
    # no query heads, and a q pointer off its 16-byte boundary
    B, nq, d = q.shape
    args = (bt.data_ptr(), lens.data_ptr(), out.data_ptr())
    assert fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), *args, B, 0, 2, d, kc.shape[2], bt.shape[1], 1, 1.0,
              None) == EBADARG
    assert fn(q.data_ptr() + 2, kc.data_ptr(), vc.data_ptr(), *args, B, nq, 2, d, kc.shape[2], bt.shape[1], 1, 1.0,
              None) == EBADARG
    assert fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr() + 8, B, nq,
              2, d, kc.shape[2], bt.shape[1], 1, 1.0, None) == EBADARG
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(big_out) == 0
