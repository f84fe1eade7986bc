"""Benchmark: asynchronous DAPO training throughput (RL trained tokens/s).

Workload: DAPO on a Qwen2.5-3B-shaped decoder (random init, bf16), staleness 3,
8 responses per prompt, random-token prompts of 64-512 tokens, forced response
lengths lognormal(7.0, 0.8) capped at 8192, Bernoulli(0.3) hashed reward,
clip-higher 0.2/0.28, AdamW lr 1e-6.  Weak scaling: 16 prompts x 8 responses
per GPU per step (128 x 8 on 8 GPUs).

* N = 1: trainer and rollout engine colocated on one GPU.
* N > 1 (torch.distributed.run, one process per GPU): N/2 trainer ranks
  (sharded data parallel) and N/2 rollout ranks.

Timing: W untimed warm-up steps, then exactly K training steps bracketed by a
barrier and torch.cuda.synchronize() on both sides, measured with CUDA events
on each rank; the reported time is the max over ranks.  Trained tokens count
prompt + response tokens of every consumed trajectory.  Inputs exceed L2.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "RL trained tokens/sec (staleness=3, 8×B200); weight-sync latency & NVLink roofline %"


def _importable(mod: str) -> bool:
    import importlib.util
    return importlib.util.find_spec(mod) is not None


def reference_arm(args) -> None:
    """Run the unmodified reference through its public entry point, if it can run here."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    why = None
    if not os.path.isdir(os.path.join(ref, "psrl")):
        why = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        try:
            import psrl.trainer.main_ppo  # noqa: F401
        except Exception as exc:
            missing = [m for m in ("ray", "hydra", "omegaconf", "verl", "transfer_queue", "nixl")
                       if not _importable(m)]
            why = (f"reference entry point psrl.trainer.main_ppo cannot be imported from baseline/_ref "
                   f"({type(exc).__name__}: {exc}); its runtime dependencies are not installed and have no "
                   f"offline wheels: {', '.join(missing)}")
    rank = int(os.environ.get("RANK", 0))
    if rank == 0:
        print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": why or "unknown"}), flush=True)


def run_colocated(args) -> dict:
    import torch

    from psrl_b200.bench.rl_bench import build_cfg
    from psrl_b200.ops import _ext
    from psrl_b200.trainer import RLTrainer
    from psrl_b200.utils import transfer
    from psrl_b200.utils.clocks import ClockSampler

    cfg = build_cfg(args, 1)
    t = RLTrainer(cfg)
    t.engine.capture_all()
    for _ in range(args.warmup):
        t.step()
    torch.cuda.synchronize()
    sampler = ClockSampler([torch.cuda.current_device()]).start()
    l0 = _ext.launches()
    b0, o0 = transfer.snapshot()
    tok0 = t.trained_tokens
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    start.record()
    metrics = []
    for _ in range(args.steps):
        metrics.append(t.step())
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    t.stop_rollout()
    b1, o1 = transfer.snapshot()
    tokens = t.trained_tokens - tok0
    return {
        "ms": ms, "wall_s": wall, "tokens": tokens, "launches": _ext.launches() - l0, "clocks": clocks,
        "h2d": (b1 - b0) / args.steps, "d2h": (o1 - o0) / args.steps, "metrics": metrics,
        "prompts_per_step": cfg.psrl.staleness_buffer_entries,
        "trajectories_per_step": cfg.psrl.staleness_buffer_entries * cfg.psrl.rollout_n,
        "parallelism": "colocated-1gpu", "api": "RLTrainer.step",
        "sync": {"pulls": int(t.instance.sync_count), "pull_s": float(t.instance.sync_time),
                 "path": "in-HBM copy trainer -> engine weights (same GPU)"},
    }


def _sync_summary(res: dict) -> dict | None:
    """Weight-sync latency over the whole run (warm-up included): the rollout
    side's wall time per pull of a new version."""
    sync = res.get("sync") or (res.get("cp") or {}).get("sync")
    if not sync or not sync.get("pulls"):
        return None
    out = {"pulls": int(sync["pulls"]), "mean_ms": round(1000.0 * float(sync["pull_s"]) / int(sync["pulls"]), 2)}
    if sync.get("copies"):
        # device time of the copy kernel alone, against 770 GB/s (measured peer copy per direction)
        # and 900 GB/s (NVLink 5 nominal per direction) per receiving GPU
        copy_ms = 1000.0 * float(sync["copy_s"]) / int(sync["copies"])
        gb = float(sync.get("bytes", 0)) / 1e9
        out.update(copy_ms=round(copy_ms, 2), bytes_per_pull=int(sync.get("bytes", 0)),
                   frac_measured_link=round(gb / 770.0 * 1000.0 / copy_ms, 3) if copy_ms else None,
                   frac_nominal_link=round(gb / 900.0 * 1000.0 / copy_ms, 3) if copy_ms else None)
    out["path"] = sync.get("path", "NVLink peer loads from the trainers' HBM stores" if "n_train" in res
                           else "in-HBM copy from the local trainer replica")
    return out


def _breakdown(metrics: list) -> dict:
    """Mean per timed step of every stage timer (``timing_s/*``) the trainer
    reports: waiting for generation, log-prob passes, the update, the push."""
    keys = sorted({k for m in metrics for k in m if k.startswith("timing_s/")})
    return {k.split("/", 1)[1]: round(sum(float(m.get(k, 0.0)) for m in metrics) / max(1, len(metrics)), 3)
            for k in keys}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="psrl_b200", choices=["psrl_b200", "reference"])
    ap.add_argument("--preset", default="dapo_qwen2.5_3b")
    ap.add_argument("--prompts-per-gpu", type=int, default=16)
    ap.add_argument("--max-num-seqs", type=int, default=512)
    ap.add_argument("--kv-cache-gb", type=float, default=32.0)
    ap.add_argument("--recompute", action="store_true",
                    help="activation recompute in the trainer (off by default: the 3B activations of a "
                         "10k-token micro-batch fit in HBM next to the KV cache)")
    ap.add_argument("--override", action="append", default=[])
    ap.add_argument("--placement", default="auto", choices=["auto", "colocated", "hybrid", "disaggregated"],
                    help="auto: colocated on one GPU; on several, disaggregated (half the GPUs train with "
                         "sharded data parallelism, half serve rollout), the 4 + 4 split of the 8-GPU "
                         "DAPO recipe")
    ap.add_argument("--stack-dump-s", type=float, default=0.0,
                    help="print every thread's stack each this many seconds (debugging stalls; 0 = off)")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.stack_dump_s > 0:
        import faulthandler
        faulthandler.dump_traceback_later(args.stack_dump_s, repeat=True)
    placement = args.placement
    if placement == "auto":
        placement = "disaggregated" if (args.gpus > 1 or world > 1) else "colocated"
    if placement != "colocated":
        from psrl_b200.trainer.distributed import run_disaggregated_bench
        res = run_disaggregated_bench(args, placement)
        if res is None:
            return
    else:
        res = run_colocated(args)
    ms_per_step = res["ms"] / args.steps
    value = res["tokens"] / (res["ms"] / 1000.0)
    e2e = res["tokens"] / res["wall_s"]
    if args.verbose:
        for m in res["metrics"]:
            print(json.dumps({k: v for k, v in m.items()}, default=str), file=sys.stderr)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "trained tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-token prompts, forced lognormal response lengths, random-init weights)",
        "config": {
            "model": "Qwen2.5-3B architecture (36L, h2048, 16Q/2KV, I11008, V151936)",
            "algorithm": "DAPO, staleness=3, 8 responses/prompt",
            "global_batch": res["prompts_per_step"],
            "prompts_per_step": res["prompts_per_step"],
            "trajectories_per_step": res["trajectories_per_step"],
            "seq_len": "prompt U[64,512] + response lognormal(7.0,0.8) cap 8192",
            "parallelism": res["parallelism"],
            "l2": "inputs larger than L2 (weights 6.2 GB, KV cache tens of GB)",
            "activation_recompute": bool(args.recompute),
        },
        "clocks": res["clocks"],
        "e2e": {"value": round(e2e, 1), "unit": f"trained tokens/s (wall clock, public API {res['api']})",
                "h2d_bytes_per_step": int(res["h2d"]), "d2h_bytes_per_step": int(res["d2h"])},
        "gpu_launches": int(res["launches"]),
        "breakdown_s_per_step": _breakdown(res["metrics"]),
        "rollout_engines": (res.get("cp") or {}).get("rollout"),
        "weight_sync": _sync_summary(res),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
