"""Debug-build bounds checks (csrc/checks.cuh).

Every bad index below still points into memory that the test allocated (the
kernel sees a VIEW of a larger cache, or a row of a larger block table), so a
regular build, which has no checks, reads valid memory and the test only
confirms that nothing is reported.  A build with PSRL_KERNEL_CHECKS=1 must
record the failure, skip the access and keep the context usable.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

D = 128


@pytest.fixture(autouse=True)
def _clean():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from psrl_b200.ops.debug import kernel_check_record
    kernel_check_record(clear=True)
    yield
    kernel_check_record(clear=True)


def _expect(code: int) -> None:
    from psrl_b200.ops.debug import CODES, check_kernel_bounds, kernel_checks_enabled
    if kernel_checks_enabled():
        with pytest.raises(RuntimeError, match=CODES[code].split(":")[0]):
            check_kernel_bounds()
    else:
        check_kernel_bounds()   # a regular build reports nothing
    assert int(torch.ones(8, device="cuda").sum().item()) == 8   # the context is usable


def _cache(n_blocks_view: int, extra: int, nkv: int = 2, bs: int = 64):
    big = torch.randn(n_blocks_view + extra, nkv, bs, D, device="cuda").bfloat16()
    return big, big[:n_blocks_view]


def test_decode_block_id_out_of_range():
    from psrl_b200.ops import paged_decode_attention
    bigk, kc = _cache(8, 4)
    bigv, vc = _cache(8, 4)
    bt = torch.arange(8, dtype=torch.int32, device="cuda").view(2, 4)
    bt[1, 2] = 9                               # past the view's 8 blocks, inside the allocation
    lens = torch.tensor([256, 256], dtype=torch.int32, device="cuda")
    q = torch.randn(2, 16, D, device="cuda").bfloat16()
    out = paged_decode_attention(q, kc, vc, bt, lens, splits=1)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    _expect(64)


def test_decode_kv_len_above_table():
    from psrl_b200.ops import paged_decode_attention
    _, kc = _cache(8, 0)
    _, vc = _cache(8, 0)
    bt = torch.arange(8, dtype=torch.int32, device="cuda").view(2, 4)
    # sequence 0 claims 5 blocks of a 4-slot row: its fifth slot is row 1's first
    lens = torch.tensor([5 * 64, 128], dtype=torch.int32, device="cuda")
    q = torch.randn(2, 16, D, device="cuda").bfloat16()
    paged_decode_attention(q, kc, vc, bt, lens, splits=1)
    torch.cuda.synchronize()
    _expect(63)


def test_prefill_block_id_out_of_range():
    from psrl_b200.ops import paged_prefill_attention
    _, kc = _cache(8, 4)
    _, vc = _cache(8, 4)
    bt = torch.arange(8, dtype=torch.int32, device="cuda").view(2, 4)
    bt[0, 1] = 10
    lens = torch.tensor([200, 100], dtype=torch.int32, device="cuda")
    cu_q = torch.tensor([0, 64, 128], dtype=torch.int32, device="cuda")
    q = torch.randn(128, 16, D, device="cuda").bfloat16()
    paged_prefill_attention(q, kc, vc, cu_q, lens, bt, 64)
    torch.cuda.synchronize()
    _expect(62)


def test_kv_copy_block_out_of_range():
    from psrl_b200.rollout.kv_offload import copy_blocks
    srck = [_cache(6, 2)[1] for _ in range(2)]
    srcv = [_cache(6, 2)[1] for _ in range(2)]
    dstk = [torch.zeros_like(t) for t in srck]
    dstv = [torch.zeros_like(t) for t in srcv]
    copy_blocks(srck, srcv, dstk, dstv, [0, 7], [1, 2])   # source block 7 is past the 6-block view
    torch.cuda.synchronize()
    torch.testing.assert_close(dstk[0][1], srck[0][0], rtol=0, atol=0)   # the valid pair was copied
    _expect(67)


def test_clean_run_reports_nothing():
    from psrl_b200.ops import check_kernel_bounds, paged_decode_attention
    _, kc = _cache(8, 0)
    _, vc = _cache(8, 0)
    bt = torch.arange(8, dtype=torch.int32, device="cuda").view(2, 4)
    lens = torch.tensor([256, 17], dtype=torch.int32, device="cuda")
    q = torch.randn(2, 16, D, device="cuda").bfloat16()
    paged_decode_attention(q, kc, vc, bt, lens)
    torch.cuda.synchronize()
    check_kernel_bounds()
