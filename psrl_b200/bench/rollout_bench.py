"""Rollout-only benchmark on the paged engine (reference: ``psrl/bench/rollout/main_rollout.py``).

Submits ``--num-requests`` random-token prompts with forced output lengths and
reports generated tokens/s, decode-step device time (CUDA events around the
engine's graph replay) vs host time, and prefill throughput.

    python -m psrl_b200.bench.rollout_bench --preset qwen2.5-3b --num-requests 256 \
        --prompt-len 256 --output-len 512
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="qwen2.5-3b")
    ap.add_argument("--num-requests", type=int, default=256)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--output-len", type=int, default=512)
    ap.add_argument("--block-size", type=int, default=64)
    ap.add_argument("--kv-cache-gb", type=float, default=40.0)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--decode-gemm", default="library", choices=["library", "tcgen05"])
    args = ap.parse_args(argv)
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams

    a = PRESETS[args.preset]
    dev = torch.device("cuda", torch.cuda.current_device())
    m = build_model(a, dev, torch.bfloat16, seed=0)
    w = EngineWeights.from_model(m)
    del m
    torch.cuda.empty_cache()
    eng = RolloutEngine(a, w, max_num_seqs=args.max_num_seqs, max_model_len=args.prompt_len + args.output_len + 64,
                        block_size=args.block_size, kv_cache_gb=args.kv_cache_gb, use_cuda_graph=not args.no_graph,
                        enable_prefix_caching=False, decode_gemm=args.decode_gemm)
    g = torch.Generator().manual_seed(0)

    def submit(base, n):
        for i in range(n):
            p = torch.randint(3, a.vocab_size, (args.prompt_len,), generator=g).tolist()
            eng.add_request(GenRequest(base + i, p, SamplingParams(max_tokens=args.output_len, ignore_eos=True,
                                                                   seed=base + i)))

    # warm-up (captures graphs for the buckets used)
    submit(10_000_000, min(args.num_requests, args.max_num_seqs))
    while eng.has_unfinished():
        eng.step()
    for k in eng.stats:
        eng.stats[k] = 0 if isinstance(eng.stats[k], int) else 0.0
    # device time of one decode-graph replay at the full batch (no host work)
    replay_ms = None
    if not args.no_graph:
        submit(20_000_000, min(args.num_requests, args.max_num_seqs))
        while eng.waiting:
            eng.step()
        eng.step()
        replay_ms = decode_step_device_time(eng)
        eng.abort_all()
    # timed
    submit(0, args.num_requests)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    n_out = 0
    while eng.has_unfinished():
        for o in eng.step():
            n_out += len(o.output_ids)
    ev1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    dev_ms = ev0.elapsed_time(ev1)
    # isolated decode-step device time at the steady batch size
    st = eng.stats
    res = {
        "preset": args.preset, "requests": args.num_requests, "prompt_len": args.prompt_len,
        "output_len": args.output_len, "gen_tokens": n_out, "wall_s": round(wall, 3),
        "device_s": round(dev_ms / 1000, 3), "gen_tok_per_s": round(n_out / wall, 1),
        "decode_steps": st["decode_steps"], "decode_host_ms_per_step": round(1000 * st["decode_time"] / max(1, st["decode_steps"]), 3),
        "prefill_tokens": st["prefill_tokens"], "prefill_s": round(st["prefill_time"], 3),
        "decode_graph_replay_ms": round(replay_ms, 3) if replay_ms else None,
    }
    print(json.dumps(res))
    return res


def decode_step_device_time(eng, iters: int = 20) -> float:
    """Device ms of one decode-graph replay at the current batch (no host work)."""
    nb = eng._bucket(len(eng.running))
    g = eng._graphs[nb]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


if __name__ == "__main__":
    main()
