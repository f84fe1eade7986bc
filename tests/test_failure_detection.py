"""Failure detection on the host (no GPU fault): the control plane stops
waiting for a buffer when a rollout instance reported a failure or went
silent, and a disaggregated run whose rollout rank leaves abruptly ends, on
every rank, in bounded time instead of hanging."""

import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_control_plane_detects_silent_and_failed_instances():
    from psrl_b200.config import load_config
    from psrl_b200.trainer.control_plane import ControlPlane
    cp = ControlPlane(load_config(preset="cpu_tiny_grpo"), vocab_size=1024, n_train=1, liveness_s=0.2)
    cp.register_instance((0, 0), 0)
    time.sleep(0.3)
    with pytest.raises(TimeoutError, match="silent instances"):
        cp._wait_ready(0, timeout_s=5)
    cp.last_seen.clear()
    cp.report_failure((1, 0), "rollout thread raised")
    with pytest.raises(RuntimeError, match="rollout instance failed"):
        cp._wait_ready(0, timeout_s=5)
    cp.shutdown()


def _worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.distributed import run_disaggregated
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "rollout.max_response_length=12", "psrl.deployment.train_ngpus=2", "++trainer.liveness_timeout_s=5",
        "++trainer.inject_rollout_exit_after_s=1.0", "psrl.staleness=1"])
    info = init_distributed("cpu", timeout_s=30)
    run_disaggregated(cfg, steps=50, warmup=0, info=info)


def test_rollout_rank_leaving_ends_the_run():
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 3, port)) for r in range(3)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    alive = [p.is_alive() for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not any(alive), alive
    assert procs[2].exitcode == 3                      # the injected exit
    assert procs[0].exitcode != 0 and procs[1].exitcode != 0   # the trainers fail, they do not hang
    assert time.monotonic() - t0 < 240
