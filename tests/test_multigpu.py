"""Two-GPU tests: CUDA-IPC weight store + peer-load pull kernel, and a short
disaggregated RL run (1 trainer rank + 1 rollout rank).  Processes are spawned
per test; every collective has a short timeout."""

import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pull_worker(rank, world, port, q):
    import faulthandler
    faulthandler.dump_traceback_later(90, repeat=True)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.parallel.weight_sync import WeightLayout, WeightPuller, WeightStore
    info = init_distributed("cuda", timeout_s=60)
    n = (1 << 24) + 64 * 7           # ~33 MB of bf16, not a power of two
    layout = WeightLayout([("w", (n,), 0)], n, torch.bfloat16)
    if rank == 0:
        src = torch.randn(n, device="cuda").bfloat16()
        store = WeightStore(layout, info.device, "hbm")
        store.publish(src, 1)
        torch.cuda.synchronize()
        box = [store.descriptor(), float(src.float().sum()), src[:1000].float().cpu()]
    else:
        box = [None, None, None]
    dist.broadcast_object_list(box, src=0)
    dist.barrier()
    if rank == 1:
        dst = torch.zeros(n, device="cuda", dtype=torch.bfloat16)
        puller = WeightPuller(layout, [box[0]], dst)
        puller.pull()
        torch.cuda.synchronize()
        ok = abs(float(dst.float().sum()) - box[1]) < 1e-3 * max(1.0, abs(box[1])) and \
            torch.equal(dst[:1000].float().cpu(), box[2])
        # timing of a full pull (bandwidth sanity)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            puller.pull()
        e1.record()
        torch.cuda.synchronize()
        gbs = 5 * n * 2 / (e0.elapsed_time(e1) / 1000) / 1e9
        q.put({"ok": bool(ok), "gbs": gbs})
    dist.barrier()
    dist.destroy_process_group()


def test_ipc_store_pull_two_gpus():
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_pull_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(150)
    codes = [p.exitcode for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    res = q.get(timeout=5)
    assert res["ok"], res
    assert res["gbs"] > 50, res      # a peer pull over NVLink, not a host bounce


def _rl_worker(rank, world, port, q):
    import faulthandler
    faulthandler.dump_traceback_later(90, repeat=True)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.distributed import run_disaggregated
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "model.preset=tiny128", "model.dtype=bf16", "trainer.device=cuda", "psrl.ps_mode=hbm",
        "rollout.cuda_graph=true", "data.kind=synthetic_tokens", "data.prompt_len_min=16", "data.prompt_len_max=64",
        "data.response_len_mu=3.0", "data.response_len_sigma=0.5", "data.response_len_cap=64",
        "reward.kind=bernoulli_hash", "rollout.ignore_eos=true"])
    info = init_distributed("cuda", timeout_s=60)
    res = run_disaggregated(cfg, steps=2, warmup=1, info=info)
    if rank == 0:
        q.put({"tokens": res["tokens"], "pulls": res["sync"]["pulls"], "ms": res["ms"],
               "steps": [m["num_trajectories"] for m in res["metrics"]]})
    dist.destroy_process_group()


def test_disaggregated_rl_two_gpus():
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(240)
    codes = [p.exitcode for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    res = q.get(timeout=5)
    assert res["steps"] == [32, 32]
    assert res["pulls"] >= 3 and res["ms"] > 0     # initial pull + at least one per step


def _hybrid_worker(rank, world, port, q):
    import faulthandler
    faulthandler.dump_traceback_later(90, repeat=True)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.hybrid import run_hybrid
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "model.preset=tiny128", "model.dtype=bf16", "trainer.device=cuda",
        "rollout.cuda_graph=true", "data.kind=synthetic_tokens", "data.prompt_len_min=16", "data.prompt_len_max=64",
        "data.response_len_mu=3.0", "data.response_len_sigma=0.5", "data.response_len_cap=64",
        "reward.kind=bernoulli_hash", "rollout.ignore_eos=true"])
    info = init_distributed("cuda", timeout_s=60)
    res = run_hybrid(cfg, steps=2, warmup=1, info=info)
    q.put({"rank": rank, "checksum": res["param_checksum"]})
    if rank == 0:
        q.put({"steps": [m["num_trajectories"] for m in res["metrics"]], "ps_version": res["cp"]["ps_version"],
               "ms": res["ms"]})
    dist.destroy_process_group()


def test_hybrid_rl_two_gpus():
    """Both GPUs train (NCCL data parallel) and serve rollout; replicas stay identical."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_hybrid_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(240)
    codes = [p.exitcode for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    items = [q.get(timeout=5) for _ in range(3)]
    sums = {d["rank"]: d["checksum"] for d in items if "checksum" in d}
    res = next(d for d in items if "steps" in d)
    assert sums[0] == sums[1]
    assert res["steps"] == [32, 32] and res["ps_version"] == 3 and res["ms"] > 0


_GPU_TINY = ["model.dtype=bf16", "trainer.device=cuda", "rollout.cuda_graph=true", "data.kind=synthetic_tokens",
             "data.prompt_len_min=16", "data.prompt_len_max=64", "data.response_len_mu=3.0",
             "data.response_len_sigma=0.5", "data.response_len_cap=64", "reward.kind=bernoulli_hash",
             "rollout.ignore_eos=true"]


def _hybrid_cfg_worker(rank, world, port, q, overrides):
    import faulthandler
    faulthandler.dump_traceback_later(150, repeat=True)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.hybrid import run_hybrid
    cfg = load_config(preset="cpu_tiny_grpo", overrides=_GPU_TINY + list(overrides))
    info = init_distributed("cuda", timeout_s=60)
    res = run_hybrid(cfg, steps=2, warmup=0, info=info)
    ms = res["metrics"]
    q.put({"rank": rank, "engine": res["engine_checksum"], "steps": [m["num_trajectories"] for m in ms],
           "vf": [m.get("critic/vf_loss") for m in ms], "kl": [m.get("actor/reward_kl_penalty") for m in ms],
           "pg": [m.get("actor/pg_loss") for m in ms]})
    dist.destroy_process_group()


def _run_hybrid_cfg(overrides):
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_hybrid_cfg_worker, args=(r, 2, port, q, overrides)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(300)
    codes = [p.exitcode for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    return sorted([q.get(timeout=5) for _ in range(2)], key=lambda d: d["rank"])


def test_hybrid_expert_parallel_moe_two_gpus():
    """MoE training step with experts sharded over two GPUs (peer-memory
    all-to-all for dispatch and combine), in-reward KL and the KL loss, both
    ranks' engines ending with the same assembled weights."""
    res = _run_hybrid_cfg(["model.preset=tiny-moe", "++actor.expert_parallel_size=2",
                           "algorithm.use_kl_in_reward=true", "actor.use_kl_loss=true",
                           "psrl.log_prob.enable_rollout_engine_log_prob=false"])
    assert res[0]["steps"] == [32, 32]
    assert all(math.isfinite(x) for x in res[0]["pg"]), res[0]["pg"]
    assert res[0]["kl"][0] is not None and abs(res[0]["kl"][0]) < 1e-6
    assert abs(res[0]["engine"] - res[1]["engine"]) <= 1e-6 * max(1.0, abs(res[0]["engine"]))


def test_hybrid_ppo_with_critic_two_gpus():
    """PPO with a critic over two GPUs: values on each rank's share, GAE
    whitened with both ranks' statistics, critic and actor updates."""
    res = _run_hybrid_cfg(["model.preset=tiny128", "critic.enable=true", "algorithm.adv_estimator=gae"])
    assert res[0]["steps"] == [32, 32]
    assert all(v is not None and math.isfinite(v) and v >= 0 for v in res[0]["vf"]), res[0]["vf"]
    assert abs(res[0]["engine"] - res[1]["engine"]) <= 1e-6 * max(1.0, abs(res[0]["engine"]))


def _peer_step_worker(rank, world, port, q):
    import faulthandler
    faulthandler.dump_traceback_later(90, repeat=True)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.parallel.fsdp import FlatShardedDP
    info = init_distributed("cuda", timeout_s=60)
    a = PRESETS["tiny128"]
    dps = []
    for peer in (False, True):
        m = build_model(a, info.device, torch.bfloat16, seed=11)
        dp = FlatShardedDP(m, dist.group.WORLD, lr=1e-3, weight_decay=0.1, max_grad_norm=1.0)
        if peer:
            assert dp.enable_peer_step()
        dps.append(dp)
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    norms = []
    for _ in range(3):
        grad = torch.randn(dps[0].total, device="cuda", generator=g) * 0.01
        for dp in dps:
            dp.flat_grad.copy_(grad)
        norms.append([float(dp.step()["grad_norm"]) for dp in dps])
    torch.cuda.synchronize()
    base, peer = dps
    diff_master = float((base.master_all - peer.master_all).abs().max())
    diff_flat = float((base.flat.float() - peer.flat.float()).abs().max())
    # every rank must hold the same full parameters after the fused all-gather
    fl = peer.flat.float().clone()
    dist.all_reduce(fl, op=dist.ReduceOp.MAX)
    same = bool(torch.equal(fl, peer.flat.float()))
    q.put({"rank": rank, "diff_master": diff_master, "diff_flat": diff_flat, "same": same, "norms": norms,
           "zeroed": float(peer.flat_grad.abs().max())})
    dist.barrier()
    dist.destroy_process_group()


def test_peer_optimizer_step_matches_nccl_two_gpus():
    """Fused peer-memory reduce-scatter + AdamW + all-gather == NCCL path."""
    _need(2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_peer_step_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(180)
    codes = [p.exitcode for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    for _ in range(2):
        r = q.get(timeout=5)
        assert r["same"], r
        assert r["zeroed"] == 0.0, r
        assert r["diff_master"] < 1e-6, r
        assert r["diff_flat"] <= 2 ** -7, r
        for nb, npeer in r["norms"]:
            assert abs(nb - npeer) <= 1e-4 * max(1.0, nb), r
