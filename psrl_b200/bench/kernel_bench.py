"""Kernel micro-benchmarks with roofline fractions.

Each case runs a kernel on inputs larger than L2 (or rotates buffers), times
it with CUDA events after warm-up, and reports achieved bandwidth / FLOP rate
as a fraction of the measured peaks (``MEASURED_PEAKS.json`` when present).

    python -m psrl_b200.bench.kernel_bench [--only decode,gemm,...]
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


def timeit(fn, iters: int = 20, warmup: int = 5) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def bench_decode(pk):
    """Paged decode attention; sweeps the split count and the K/V ring depth
    (2 stages x 3 CTAs/SM vs 3 stages x 2 CTAs/SM).  Rollout-like cases first:
    a short-context batch and a B=512 batch at the mean in-flight context of
    lognormal(7.0, 0.8) responses."""
    from psrl_b200.ops import paged_decode_attention
    from psrl_b200.ops.attention import decode_splits
    out = []
    for B, ctx, nq, nkv in ((256, 320, 16, 2), (512, 1728, 16, 2), (256, 1024, 16, 2), (128, 4096, 16, 2),
                            (64, 8192, 28, 4)):
        bs, d = 64, 128
        nblk = B * (ctx // bs)
        kc = torch.randn(nblk, nkv, bs, d, device="cuda").bfloat16()
        vc = torch.randn_like(kc)
        # scattered pages, as the block manager hands them out
        bt = torch.randperm(nblk, device="cuda").to(torch.int32).view(B, ctx // bs)
        lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(B, nq, d, device="cuda").bfloat16()
        sp = decode_splits(B, nkv, ctx)
        nbytes = 2 * B * ctx * nkv * d * 2
        sweep = {}
        for st in (2, 3):
            for s_ in sorted({1, 2, 4, sp}):
                ms_ = timeit(lambda: paged_decode_attention(q, kc, vc, bt, lens, splits=s_, stages=st))
                sweep[f"st{st}/sp{s_}"] = round(nbytes / (ms_ / 1e3) / 1e9, 1)
        ms = timeit(lambda: paged_decode_attention(q, kc, vc, bt, lens, splits=sp))
        gbs = nbytes / (ms / 1e3) / 1e9
        bt_c = torch.arange(nblk, dtype=torch.int32, device="cuda").view(B, ctx // bs)
        ms_c = timeit(lambda: paged_decode_attention(q, kc, vc, bt_c, lens, splits=sp))
        out.append({"case": f"decode B={B} ctx={ctx} {nq}/{nkv}", "ms": round(ms, 4), "GB/s": round(gbs, 1),
                    "frac_hbm": round(gbs / pk["hbm_gbs"], 3), "splits": sp, "GB/s_by_stages_splits": sweep,
                    "GB/s_contiguous_pages": round(nbytes / (ms_c / 1e3) / 1e9, 1)})
        del kc, vc
    return out


def bench_gemm(pk):
    """Projection GEMMs of a Qwen2.5-3B training micro-batch (10240 tokens):
    the paired-CTA tcgen05 kernel in all three roles (forward x W^T, data
    gradient dy W, weight gradient dy^T x) against cuBLAS through torch on the
    same operands, plus the fused gate_up + SwiGLU epilogue."""
    from psrl_b200.ops import ext
    from psrl_b200.ops.gemm import check_errors
    from psrl_b200.ops.linear import gate_up_swiglu, matmul_nt, weight_grad
    out = []
    M = 10240
    for name, N, K in (("qkv", 2560, 2048), ("o", 2048, 2048), ("gate_up", 22016, 2048), ("down", 2048, 11008)):
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        dy = torch.randn(M, N, device="cuda").bfloat16()
        fl = 2.0 * M * N * K
        rows = {}
        for role, tc, cb in (("fwd", lambda: matmul_nt(x, w), lambda: x @ w.t()),
                             ("dgrad", lambda: matmul_nt(dy, w, b_mn=True), lambda: dy @ w),
                             ("wgrad", lambda: weight_grad(dy, x), lambda: dy.t() @ x)):
            ms_tc = timeit(tc, iters=10)
            ms_cb = timeit(cb, iters=10)
            rows[role] = {"tcgen05_ms": round(ms_tc, 3), "cublas_ms": round(ms_cb, 3),
                          "tcgen05_tflops": round(fl / ms_tc / 1e9, 1), "cublas_tflops": round(fl / ms_cb / 1e9, 1),
                          "frac_peak_tcgen05": round(fl / ms_tc / 1e9 / pk["bf16_tflops"], 3),
                          "vs_cublas": round(ms_cb / ms_tc, 3)}
        if name == "gate_up":
            ms_f = timeit(lambda: gate_up_swiglu(x, w), iters=10)
            ms_u = timeit(lambda: ext().swiglu_fwd(x @ w.t()), iters=10)
            rows["fwd+swiglu"] = {"fused_ms": round(ms_f, 3), "cublas_then_swiglu_ms": round(ms_u, 3),
                                  "vs_unfused": round(ms_u / ms_f, 3)}
        check_errors()
        out.append({"case": f"{name} M={M} N={N} K={K}", **rows})
        del x, w, dy
    return out


def _graph_time(fns, reps: int = 5) -> float:
    """Mean device time of one call of ``fns`` (a list of closures, run in
    turn) replayed from a CUDA graph, as the rollout engine runs them."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (reps * len(fns))


def bench_decode_gemm(pk):
    """Decode-step projections of the Qwen2.5-3B engine (B rows = sequences in
    the batch): the weight-streaming tcgen05 kernel against cuBLAS through torch, both
    replayed from CUDA graphs over enough weight copies that every call streams
    its weight from HBM (more than the 126 MB L2).  gate_up is timed with its
    activation: the fused SwiGLU epilogue against cuBLAS + the SwiGLU kernel.
    Reported as weight bandwidth (the bytes a decode step must stream)."""
    from psrl_b200.ops import swiglu
    from psrl_b200.ops.linear import decode_gate_up_swiglu, decode_linear
    out = []
    shapes = (("qkv", 2560, 2048), ("o", 2048, 2048), ("gate_up+swiglu", 22016, 2048), ("down", 2048, 11008),
              ("lm_head", 151936, 2048))
    for B in (16, 64, 128, 256):
        for name, N, K in shapes:
            wb = N * K * 2
            copies = max(2, -(-300_000_000 // wb))
            x = torch.randn(B, K, device="cuda").bfloat16()
            ws_ = [(torch.randn(N, K, device="cuda") * 0.02).bfloat16() for _ in range(copies)]
            if name.startswith("gate_up"):
                tc = [lambda w=w: decode_gate_up_swiglu(x, w) for w in ws_]
                cb = [lambda w=w: swiglu(x @ w.t()) for w in ws_]
            else:
                tc = [lambda w=w: decode_linear(x, w) for w in ws_]
                cb = [lambda w=w: x @ w.t() for w in ws_]
            ms_tc, ms_cb = _graph_time(tc), _graph_time(cb)
            out.append({"case": f"decode {name} B={B} N={N} K={K}", "tcgen05_us": round(ms_tc * 1e3, 1),
                        "cublas_us": round(ms_cb * 1e3, 1), "vs_cublas": round(ms_cb / ms_tc, 3),
                        "weight_GB/s_tcgen05": round(wb / ms_tc / 1e6, 1),
                        "frac_hbm_tcgen05": round(wb / ms_tc / 1e6 / pk["hbm_gbs"], 3)})
            del x, ws_
    return out


def bench_logprob(pk):
    from psrl_b200.ops.gemm import tc_linear_logprob
    from psrl_b200.ops.logprob import linear_logprob
    out = []
    T, H, V = 8192, 2048, 151936
    h = (torch.randn(T, H, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(V, H, device="cuda") * 0.02).bfloat16()
    lab = torch.randint(0, V, (T,), device="cuda")
    fl = 2.0 * T * V * H
    ms_f = timeit(lambda: tc_linear_logprob(h, w, lab), iters=10)
    with torch.no_grad():
        ms_c = timeit(lambda: linear_logprob(h, w, lab), iters=10)
    out.append({"case": f"lm-head logprob T={T} V={V}", "fused_tcgen05_ms": round(ms_f, 3),
                "cublas+lse_kernel_ms": round(ms_c, 3), "fused_tflops": round(fl / ms_f / 1e9, 1),
                "frac_peak": round(fl / ms_f / 1e9 / pk["bf16_tflops"], 3)})
    return out


def bench_attn_train(pk):
    from psrl_b200.ops import varlen_attention
    out = []
    for L, nseq in ((1700, 6), (2048, 5), (8192, 1)):
        nq, nkv, d = 16, 2, 128
        T = L * nseq
        qkv = torch.randn(T, (nq + 2 * nkv) * d, device="cuda").bfloat16().requires_grad_(True)
        cu = torch.arange(0, T + 1, L, dtype=torch.int32, device="cuda")   # nseq sequences of L tokens
        fl = 4.0 * nseq * (L * L / 2) * d * nq
        ms_f = timeit(lambda: varlen_attention(qkv, cu, L, nq, nkv, d), iters=10)
        from psrl_b200.ops import ext
        q = qkv.detach()[:, : nq * d].view(T, nq, d)
        k = qkv.detach()[:, nq * d:(nq + nkv) * d].view(T, nkv, d)
        v = qkv.detach()[:, (nq + nkv) * d:].view(T, nkv, d)
        ms_f_old = timeit(lambda: ext().attn_varlen_fwd(q, k, v, cu, L, 1 / math.sqrt(d), True), iters=10)
        o = varlen_attention(qkv, cu, L, nq, nkv, d)
        g = torch.randn_like(o)
        ms_b = timeit(lambda: torch.autograd.grad(o, qkv, g, retain_graph=True), iters=10)
        out.append({"case": f"varlen attn L={L}x{nseq} 16/2", "fwd_ms": round(ms_f, 3), "bwd_ms": round(ms_b, 3),
                    "fwd_tflops": round(fl / ms_f / 1e9, 1), "bwd_tflops": round(2.5 * fl / ms_b / 1e9, 1),
                    "fwd_frac_peak": round(fl / ms_f / 1e9 / pk["bf16_tflops"], 3),
                    "fwd_mma_sync_ms": round(ms_f_old, 3), "fwd_vs_mma_sync": round(ms_f_old / ms_f, 2)})
    return out


def bench_elementwise(pk):
    from psrl_b200.ops import rms_norm, swiglu
    out = []
    T, h, I = 65536, 2048, 11008
    x = torch.randn(T, h, device="cuda").bfloat16()
    r = torch.randn_like(x)
    w = torch.ones(h, device="cuda").bfloat16()
    with torch.no_grad():
        ms = timeit(lambda: rms_norm(x, w, 1e-6, r))
    nb = 4 * T * h * 2
    out.append({"case": f"rmsnorm+residual {T}x{h}", "ms": round(ms, 4), "GB/s": round(nb / ms / 1e6, 1),
                "frac_hbm": round(nb / ms / 1e6 / pk["hbm_gbs"], 3)})
    gu = torch.randn(16384, 2 * I, device="cuda").bfloat16()
    with torch.no_grad():
        ms = timeit(lambda: swiglu(gu))
    nb = 16384 * 3 * I * 2
    out.append({"case": f"swiglu 16384x{I}", "ms": round(ms, 4), "GB/s": round(nb / ms / 1e6, 1),
                "frac_hbm": round(nb / ms / 1e6 / pk["hbm_gbs"], 3)})
    return out


def bench_sync(pk):
    from psrl_b200.ops import ext
    n = 3_300_000_000 // 2
    src = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    dst = torch.empty_like(src)
    nb = n * 2
    ms = timeit(lambda: ext().copy_segments(dst, [src], [0], [0], [nb]), iters=10)
    return [{"case": "weight store publish (local copy_segments, 3.3 GB)", "ms": round(ms, 3),
             "GB/s (read+write)": round(2 * nb / ms / 1e6, 1), "frac_hbm": round(2 * nb / ms / 1e6 / pk["hbm_gbs"], 3)}]


def bench_sample(pk):
    """Fused Gumbel-max sampler over a [B, 151936] bf16 logits batch (one read
    of the logits is the floor)."""
    from psrl_b200.ops import sample
    out = []
    for B in (256, 512):
        V = 151936
        logits = torch.randn(B, V, device="cuda").bfloat16()
        temps = torch.ones(B, device="cuda")
        seeds = torch.arange(B, device="cuda")
        streams = torch.zeros(B, device="cuda", dtype=torch.int32)
        ms = timeit(lambda: sample(logits, temps, seeds, streams))
        gbs = B * V * 2 / (ms / 1e3) / 1e9
        out.append({"case": f"sample B={B} V={V}", "ms": round(ms, 4), "GB/s": round(gbs, 1),
                    "frac_hbm": round(gbs / pk["hbm_gbs"], 3)})
    return out


def bench_train_mb(pk):
    """One trainer micro-batch of the DAPO 3B workload: 6 sequences x 1700
    tokens (10.2k tokens) through the Qwen2.5-3B decoder, forward + backward
    of the fused LM-head log-prob, no activation recompute.  2 warm-up + 3
    timed iterations (5 in total, so a launch-list capture of the whole run
    shows each kernel 5 times)."""
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.trainer.batch import Trajectory, build_micro_batch
    a = PRESETS["qwen2.5-3b"]
    model = build_model(a, torch.device("cuda"), torch.bfloat16, seed=0)
    g = torch.Generator().manual_seed(0)
    trajs = []
    for i in range(6):
        toks = torch.randint(3, a.vocab_size, (1700,), generator=g).tolist()
        trajs.append(Trajectory(uid=i, request_id=i, prompt_ids=toks[:200], response_ids=toks[200:],
                                rollout_logprobs=[0.0] * 1500, old_logprobs=[0.0] * 1500, advantage=1.0))
    mb = build_micro_batch(trajs, list(range(6)), torch.device("cuda"))

    def run():
        lp, ent = model.logprobs(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen, mb.labels)
        (lp.sum() * 1e-6 + ent.sum() * 1e-9).backward()

    ms = timeit(run, iters=3, warmup=2)
    # one more iteration inside a "train_mb" NVTX range on both the launching
    # thread (forward) and the autograd thread (backward: pushed when the loss
    # gradient starts flowing, popped after the embedding's last gradient
    # accumulation), for launch-list captures with --nvtx-include "train_mb/"
    nvtx = torch.cuda.nvtx
    emb = model.embed.weight
    def _pop(_p):
        nvtx.range_pop()

    hook = emb.register_post_accumulate_grad_hook(_pop)
    nvtx.range_push("train_mb")
    lp, ent = model.logprobs(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen, mb.labels)
    loss = lp.sum() * 1e-6 + ent.sum() * 1e-9
    nvtx.range_pop()
    def _push(g):
        nvtx.range_push("train_mb")
        return g

    loss.register_hook(_push)
    loss.backward()
    hook.remove()
    torch.cuda.synchronize()
    T = mb.input_ids.numel()
    # matmul FLOPs (6 x params x tokens, LM head included) + causal attention (fwd 1x, bwd 2.5x)
    n_params = sum(p.numel() for p in model.parameters())
    fl = 6.0 * n_params * T + 3.5 * 4.0 * a.num_layers * a.num_heads * a.head_dim * sum(
        (1700 * 1700) / 2 for _ in range(6))
    del model
    return [{"case": f"train micro-batch qwen2.5-3b 6x1700 tokens fwd+bwd", "ms": round(ms, 2),
             "tok_per_s": round(T / ms * 1e3, 0), "tflops": round(fl / ms / 1e9, 1),
             "frac_bf16": round(fl / ms / 1e9 / pk["bf16_tflops"], 3)}]


CASES = {"decode_gemm": bench_decode_gemm, "train_mb": bench_train_mb, "sample": bench_sample, "decode": bench_decode, "gemm": bench_gemm, "logprob": bench_logprob, "attn": bench_attn_train,
         "elementwise": bench_elementwise, "sync": bench_sync}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=",".join(CASES))
    args = ap.parse_args(argv)
    pk = peaks()
    res = {"peaks": pk}
    for name in args.only.split(","):
        res[name] = CASES[name](pk)
        print(json.dumps({name: res[name]}), flush=True)
        torch.cuda.empty_cache()
    return res


if __name__ == "__main__":
    main()
