"""Command-line entry point (C1).

    python -m psrl_b200.trainer.main --preset dapo_qwen2.5_3b [--config my.yaml] \
        psrl.staleness=3 ++trainer.total_training_steps=100

One process runs colocated (trainer + rollout on one device).  Under
``torch.distributed.run`` (one process per GPU, rendezvous on 127.0.0.1)
``psrl.deployment.placement`` selects ``disaggregated`` (ranks split into
trainer and rollout roles, :mod:`.distributed`) or ``hybrid`` (every rank
trains and serves rollout, :mod:`.hybrid`).
"""

from __future__ import annotations

import argparse
import json
import os
import sys


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="psrl_b200")
    ap.add_argument("--config", default=None, help="YAML merged over the defaults/preset")
    ap.add_argument("--preset", default=None)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--print-config", action="store_true")
    ap.add_argument("overrides", nargs="*", help="key=value / ++key=value")
    args = ap.parse_args(argv)
    from ..config import load_config
    cfg = load_config(args.config, args.overrides, preset=args.preset)
    if args.print_config:
        print(cfg.to_yaml())
        return 0
    # without --steps: trainer.total_training_steps counts from step 0, so a
    # resumed run does only the steps still missing
    steps = args.steps
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1:
        from ..parallel.dist import destroy, init_distributed
        info = init_distributed(cfg.trainer.get("device", "auto"))
        if cfg.psrl.deployment.get("placement", "disaggregated") == "hybrid":
            from .hybrid import run_hybrid
            res = run_hybrid(cfg, steps=steps, warmup=0, info=info)
        else:
            from .distributed import run_disaggregated
            res = run_disaggregated(cfg, steps=steps, warmup=0, info=info)
        if info.rank == 0:
            for m in res["metrics"]:
                print(json.dumps(m, default=str), flush=True)
        destroy()
        return 0
    from .driver import RLTrainer
    t = RLTrainer(cfg)
    for m in t.fit(steps):
        print(json.dumps({k: v for k, v in m.items() if not k.startswith("rollout/")}, default=str), flush=True)
    t.stop_rollout()
    return 0


if __name__ == "__main__":
    sys.exit(main())
