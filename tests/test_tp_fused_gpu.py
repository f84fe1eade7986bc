"""Tensor-parallel GEMMs fused with their all-reduce (csrc/gemm_2sm.cu
OUT_F32_ADD2, csrc/tp_fused.cu) against fp32 references and against the
unfused local-GEMM + NCCL all-reduce path, on two GPUs; and the cross-GPU flag
barrier's bounded wait on one GPU (a peer that never arrives: the kernel
returns an error status, the context stays usable)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                          LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        from psrl_b200.ops.gemm import check_errors
        from psrl_b200.parallel.tp_fused import FusedTP, column_parallel, row_parallel
        grp = dist.new_group([0, 1])
        ftp = FusedTP(grp, dev, max_elems=2048 * 1024)
        out = {}
        # 1) y = sum over ranks of x_r W_r^T, three calls in a row (both accumulators reused)
        for call, (M, K, N) in enumerate(((1000, 896, 1024), (2048, 512, 1024), (300, 1024, 512))):
            g = torch.Generator(device=dev).manual_seed(100 * call + rank)
            x = torch.randn(M, K, device=dev, generator=g).bfloat16()
            w = (torch.randn(N, K, device=dev, generator=g) * 0.05).bfloat16()
            y = ftp.gemm_allreduce(x, w)
            torch.cuda.synchronize()
            check_errors(dev)
            part = x.float() @ w.float().t()
            ref = part.clone()
            dist.all_reduce(ref, group=grp)
            err = (y.float() - ref).abs().max().item()
            out[f"fwd{call}"] = err / max(1.0, ref.abs().max().item())
            ys = [torch.empty_like(y) for _ in range(2)]
            dist.all_gather(ys, y, group=grp)
            out[f"same{call}"] = bool(torch.equal(ys[0], ys[1]))
        # 2) autograd: row- and column-parallel against fp32 with an NCCL all-reduce
        g = torch.Generator(device=dev).manual_seed(7 + rank)
        x0 = torch.randn(777, 512, device=dev, generator=g).bfloat16()
        wc = (torch.randn(256, 512, device=dev, generator=g) * 0.05).bfloat16()   # column-parallel shard
        wr = (torch.randn(512, 256, device=dev, generator=g) * 0.05).bfloat16()   # row-parallel shard
        dy = torch.randn(777, 512, device=dev, generator=torch.Generator(device=dev).manual_seed(99)).bfloat16()
        x = x0.clone().requires_grad_(True)
        pc, pr = wc.clone().requires_grad_(True), wr.clone().requires_grad_(True)
        y = row_parallel(column_parallel(x, pc, None, ftp), pr, ftp)
        y.backward(dy)
        torch.cuda.synchronize()
        check_errors(dev)
        xf = x0.float().requires_grad_(True)
        cf, rf = wc.float().requires_grad_(True), wr.float().requires_grad_(True)
        yp = (xf @ cf.t()) @ rf.t()
        yr = yp.detach().clone()
        dist.all_reduce(yr, group=grp)
        yp.backward(dy.float())
        dx = xf.grad.clone()
        dist.all_reduce(dx, group=grp)
        for name, got, want in (("y", y.float(), yr), ("dx", x.grad.float(), dx), ("dwc", pc.grad.float(), cf.grad),
                                ("dwr", pr.grad.float(), rf.grad)):
            out[name] = (got - want).abs().max().item() / max(1.0, want.abs().max().item())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as exc:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, {"error": f"{exc}\n{traceback.format_exc()}"}))


def test_fused_tp_gemm_allreduce_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, out in res.items():
        assert "error" not in out, out.get("error")
        for k, v in out.items():
            if k.startswith("same"):
                assert v, f"rank {r}: ranks hold different sums ({k})"
            else:
                assert v < 3e-2, f"rank {r}: {k} relative error {v}"


def test_peer_barrier_times_out_with_error_status():
    """A peer that never arrives: the barrier kernel gives up after its bound,
    records error 51 with the missing rank, and the GPU keeps working."""
    from psrl_b200.ops import ext
    from psrl_b200.ops.gemm import _err, check_errors
    dev = torch.device("cuda", 0)
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    slot_in = [flags[0:1], flags[16:17]]          # "our" slot in both arrays (both local here)
    own = [flags[0:1], flags[32:33]]              # rank 1's slot: nothing ever writes it
    err = _err(dev)
    ext().peer_barrier(slot_in, own, 1, 0.2, err)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="flag barrier timed out"):
        check_errors(dev)
    # the context is still usable
    assert int(torch.ones(4, device=dev).sum().item()) == 4
