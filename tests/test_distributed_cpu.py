"""CPU/gloo world_size=2 plumbing run: rank 0 trainer (+PS, dispatcher), rank 1
rollout; weight sync through the shared-memory Parameter Server store; GRPO at
staleness=1 on the 2-layer Qwen2-style decoder; seeded additions; 8 prompts x 4
samples per step for 4 steps."""

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(2)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.distributed import run_disaggregated
    cfg = load_config(preset="cpu_tiny_grpo")
    info = init_distributed("cpu", timeout_s=300)
    res = run_disaggregated(cfg, steps=4, warmup=0, info=info)
    if rank == 0:
        q.put({k: res[k] for k in ("tokens", "sync", "manager", "n_train", "world")} |
              {"steps": [(m["step"], m["num_trajectories"]) for m in res["metrics"]]})
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gloo_world2_plumbing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    res = q.get(timeout=5)
    assert res["n_train"] == 1 and res["world"] == 2
    assert res["steps"] == [(0, 32), (1, 32), (2, 32), (3, 32)]
    assert res["tokens"] > 0
    assert res["sync"]["pulls"] >= 2      # initial pull + at least one newer version


def _worker4(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.distributed import run_disaggregated
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12",
                                                         "psrl.deployment.train_ngpus=2"])
    info = init_distributed("cpu", timeout_s=300)
    res = run_disaggregated(cfg, steps=2, warmup=1, info=info)
    if rank == 0:
        q.put({"n_train": res["n_train"], "steps": [m["num_trajectories"] for m in res["metrics"]],
               "pulls": res["sync"]["pulls"]})
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gloo_world4_two_trainers_two_rollouts():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker4, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0, 0, 0], codes
    res = q.get(timeout=5)
    assert res["n_train"] == 2 and res["steps"] == [32, 32]
    # each rollout instance: the initial pull plus at least one newer version
    # (an instance that sees two new versions at once pulls only the latest)
    assert res["pulls"] >= 2 * 2


def _worker_hybrid(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.hybrid import run_hybrid
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12"])
    info = init_distributed("cpu", timeout_s=300)
    res = run_hybrid(cfg, steps=2, warmup=1, info=info)
    q.put({"rank": rank, "checksum": res["param_checksum"]})
    if rank == 0:
        q.put({"steps": [m["num_trajectories"] for m in res["metrics"]], "tokens": res["tokens"],
               "pulls": res["cp"]["sync"]["pulls"], "ps_version": res["cp"]["ps_version"]})
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gloo_world2_hybrid_placement():
    """Every rank trains (data parallel over gloo) and serves a rollout instance;
    the control plane runs in its own process."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_hybrid, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    items = [q.get(timeout=5) for _ in range(3)]
    sums = {d["rank"]: d["checksum"] for d in items if "checksum" in d}
    res = next(d for d in items if "steps" in d)
    assert sums[0] == sums[1]         # identical replicas after the data-parallel steps
    assert res["steps"] == [32, 32] and res["tokens"] > 0
    assert res["ps_version"] == 3
    assert res["pulls"] >= 2          # both engines picked up at least one new version


def test_gloo_world4_hybrid_placement():
    """Four ranks, each a trainer replica and a rollout instance."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_hybrid, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0, 0, 0], codes
    items = [q.get(timeout=5) for _ in range(5)]
    sums = {d["rank"]: d["checksum"] for d in items if "checksum" in d}
    res = next(d for d in items if "steps" in d)
    assert len(set(sums.values())) == 1, sums
    assert res["steps"] == [32, 32] and res["ps_version"] == 3


def _worker_hybrid_ppo(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.hybrid import run_hybrid
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12", "critic.enable=true",
                                                         "algorithm.adv_estimator=gae"])
    info = init_distributed("cpu", timeout_s=300)
    res = run_hybrid(cfg, steps=2, warmup=0, info=info)
    if rank == 0:
        q.put({"steps": [m["num_trajectories"] for m in res["metrics"]],
               "vf": [m.get("critic/vf_loss") for m in res["metrics"]]})
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gloo_world2_hybrid_ppo_with_critic():
    """PPO with a critic in the hybrid placement: values on each rank's share,
    GAE whitened with all ranks' statistics, critic and actor updates."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_hybrid_ppo, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    res = q.get(timeout=5)
    assert res["steps"] == [32, 32]
    assert all(v is not None and v >= 0 for v in res["vf"]), res


def _worker_hybrid_sharded(rank, world, port, q, overrides):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.hybrid import run_hybrid
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12"] + list(overrides))
    info = init_distributed("cpu", timeout_s=300)
    res = run_hybrid(cfg, steps=2, warmup=0, info=info)
    q.put({"rank": rank, "engine": res["engine_checksum"], "tokens": res["tokens"],
           "steps": [m["num_trajectories"] for m in res["metrics"]] if rank == 0 else None,
           "kl": [m.get("actor/reward_kl_penalty") for m in res["metrics"]] if rank == 0 else None,
           "kl_coef": [m.get("actor/reward_kl_penalty_coeff") for m in res["metrics"]] if rank == 0 else None,
           "chunks": [m.get("fine_grain/chunks") for m in res["metrics"]] if rank == 0 else None,
           "pre": [m.get("fine_grain/precomputed") for m in res["metrics"]] if rank == 0 else None,
           "val": [m.get("val/num_samples") for m in res["metrics"]] if rank == 0 else None,
           "step_ids": [m.get("step") for m in res["metrics"]] if rank == 0 else None})
    import torch.distributed as dist
    dist.destroy_process_group()


def _run_sharded(overrides):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_hybrid_sharded, args=(r, 2, port, q, overrides)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    return sorted([q.get(timeout=5) for _ in range(2)], key=lambda d: d["rank"])


def test_gloo_world2_hybrid_checkpoint_resume(tmp_path):
    """The hybrid placement saves every step and a new run resumes after the
    last saved step."""
    d = str(tmp_path / "ckpt")
    first = _run_sharded([f"trainer.default_local_dir={d}", "trainer.save_freq=1"])
    assert first[0]["step_ids"] == [0, 1]
    again = _run_sharded([f"trainer.default_local_dir={d}", "trainer.resume_mode=auto"])
    assert again[0]["step_ids"] == [2, 3] and again[0]["steps"] == [32, 32]


def test_gloo_world2_hybrid_validation():
    """trainer.test_freq=1 in the hybrid placement: validation samples run on
    the ranks' engines between steps and stay out of the training buffers."""
    res = _run_sharded(["trainer.test_freq=1", "++data.val_size=4"])
    assert res[0]["steps"] == [32, 32]
    assert res[0]["val"] == [4, 4], res[0]


def test_gloo_world2_hybrid_expert_parallel_moe():
    """MoE trainer with experts sharded over two ranks; both full-model
    engines receive identical assembled weights."""
    res = _run_sharded(["model.preset=tiny-moe", "++actor.expert_parallel_size=2"])
    assert res[0]["steps"] == [32, 32]
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"]))


@pytest.mark.parametrize("rollout_tp", [1, 2])
def test_gloo_world2_hybrid_expert_tensor_parallel_moe(rollout_tp):
    """MoE trainer at TP=2 with every expert split along its width; the
    engines take the assembled full model (rollout TP 1) or the trainer's own
    shards (rollout TP 2, the engine then runs width-split experts)."""
    res = _run_sharded(["model.preset=tiny-moe", "++actor.tensor_parallel_size=2",
                        f"rollout.tensor_parallel_size={rollout_tp}"])
    assert res[0]["steps"] == [32, 32]
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"])) or rollout_tp > 1


def test_gloo_world2_hybrid_expert_parallel_in_reward_kl():
    """MoE at EP=2 with in-reward KL (adaptive coefficient), the KL loss and
    trainer-side old log-probs, with a token budget small enough that the two
    ranks pack different numbers of micro-batches (expert-parallel forwards
    stay in lockstep)."""
    res = _run_sharded(["model.preset=tiny-moe", "++actor.expert_parallel_size=2",
                        "algorithm.use_kl_in_reward=true", "algorithm.kl_ctrl.type=adaptive",
                        "actor.use_kl_loss=true", "psrl.log_prob.enable_rollout_engine_log_prob=false",
                        "actor.ppo_max_token_len_per_gpu=160"])
    assert res[0]["steps"] == [32, 32]
    kl, coef = res[0]["kl"], res[0]["kl_coef"]
    assert kl[0] is not None and abs(kl[0]) < 1e-6, kl       # step 0: actor == reference
    assert kl[1] is not None and kl[1] == kl[1], kl
    assert coef[0] == 0.001 and coef[1] < coef[0], coef      # adaptive: KL below target lowers beta
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"]))


def test_gloo_world2_hybrid_rollout_correction():
    """Trainer-side old log-probs with sequence IS weights and token
    rejection sampling; the loss normaliser is recounted over both ranks."""
    res = _run_sharded(["psrl.log_prob.enable_rollout_engine_log_prob=false",
                        "algorithm.rollout_correction.rollout_is=sequence",
                        "algorithm.rollout_correction.rollout_rs=token"])
    assert res[0]["steps"] == [32, 32]
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"]))


def test_gloo_world2_hybrid_fine_grain_per_sample_overlap():
    """Old and reference log-probs computed chunk by chunk while the buffer
    fills (posted to the control plane), with the KL loss on."""
    res = _run_sharded(["psrl.log_prob.enable_rollout_engine_log_prob=false", "actor.use_kl_loss=true",
                        "psrl.fine_grain_overlap.granularity=micro_batch", "psrl.fine_grain_overlap.multiplier=2"])
    assert res[0]["steps"] == [32, 32]
    assert all(c is not None and c >= 1 for c in res[0]["chunks"]), res[0]["chunks"]
    assert all(p is not None and p > 0 for p in res[0]["pre"]), res[0]["pre"]
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"]))


def test_gloo_world2_hybrid_pre_step_overlap():
    """Each committed mini-batch is trained (its own optimizer step) while
    the buffer fills, with trainer-side old log-probs; both engines end with
    the same weights."""
    res = _run_sharded(["psrl.log_prob.enable_rollout_engine_log_prob=false",
                        "psrl.fine_grain_overlap.granularity=mini_batch", "psrl.fine_grain_overlap.overlap_scope=pre_step",
                        "actor.ppo_mini_batch_size=4", "psrl.staleness_buffer_entries=8"])
    assert res[0]["steps"] == [32, 32]
    assert all(c is not None and c >= 2 for c in res[0]["chunks"]), res[0]["chunks"]
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"]))


def test_gloo_world2_hybrid_tensor_parallel():
    """Dense trainer at TP=2 (one data-parallel rank); both engines hold the
    assembled full weights."""
    res = _run_sharded(["++actor.tensor_parallel_size=2"])
    assert res[0]["steps"] == [32, 32]
    assert abs(res[0]["engine"] - res[1]["engine"]) < 1e-6 * max(1.0, abs(res[0]["engine"]))


def _worker_disagg_sharded(rank, world, port, q, overrides):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    torch.set_num_threads(1)
    from psrl_b200.config import load_config
    from psrl_b200.parallel.dist import init_distributed
    from psrl_b200.trainer.distributed import run_disaggregated
    cfg = load_config(preset="cpu_tiny_grpo", overrides=["rollout.max_response_length=12",
                                                         "psrl.deployment.train_ngpus=2"] + list(overrides))
    info = init_distributed("cpu", timeout_s=300)
    res = run_disaggregated(cfg, steps=2, warmup=0, info=info)
    if rank == 0:
        q.put({"steps": [m["num_trajectories"] for m in res["metrics"]], "pulls": res["sync"]["pulls"],
               "val": [m.get("val/num_samples") for m in res["metrics"]],
               "step_ids": [m.get("step") for m in res["metrics"]],
               "pre": [m.get("fine_grain/precomputed") for m in res["metrics"]],
               "kl": [m.get("actor/reward_kl_penalty") for m in res["metrics"]],
               "chunks": [m.get("fine_grain/chunks") for m in res["metrics"]]})
    import torch.distributed as dist
    dist.destroy_process_group()


def test_gloo_world3_disaggregated_tensor_parallel_trainer():
    """Two trainer ranks at TP=2 publish the assembled full model; one rollout rank pulls it."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_disagg_sharded, args=(r, 3, port, q, ["++actor.tensor_parallel_size=2"]))
             for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0, 0], codes
    res = q.get(timeout=5)
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world3_disaggregated_ppo_with_critic():
    """PPO with a critic in the disaggregated placement (two trainer ranks, one rollout rank)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ov = ["critic.enable=true", "algorithm.adv_estimator=gae"]
    procs = [ctx.Process(target=_worker_disagg_sharded, args=(r, 3, port, q, ov)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0, 0], codes
    assert q.get(timeout=5)["steps"] == [32, 32]


def test_gloo_world3_disaggregated_critic_kl_in_reward_fine_grain():
    """Disaggregated PPO with a critic, in-reward KL against a reference model
    and per-sample stages (old / reference log-probs, values) overlapped with
    the buffer filling."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ov = ["critic.enable=true", "algorithm.adv_estimator=gae", "algorithm.use_kl_in_reward=true",
          "psrl.log_prob.enable_rollout_engine_log_prob=false", "psrl.fine_grain_overlap.granularity=mini_batch"]
    procs = [ctx.Process(target=_worker_disagg_sharded, args=(r, 3, port, q, ov)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0, 0], codes
    res = q.get(timeout=5)
    assert res["steps"] == [32, 32]
    assert all(p is not None and p > 0 for p in res["pre"]), res
    assert all(k is not None for k in res["kl"]), res


def test_gloo_world3_disaggregated_pre_step_overlap():
    """Two trainer ranks train each committed mini-batch while the rollout
    rank keeps filling the buffer."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ov = ["psrl.fine_grain_overlap.granularity=mini_batch", "psrl.fine_grain_overlap.overlap_scope=pre_step",
          "actor.ppo_mini_batch_size=4"]
    procs = [ctx.Process(target=_worker_disagg_sharded, args=(r, 3, port, q, ov)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0, 0], codes
    res = q.get(timeout=5)
    assert res["steps"] == [32, 32] and all(c == 2 for c in res["chunks"]), res


def test_multi_gpu_pre_step_rejects_batch_statistics():
    import pytest

    from psrl_b200.config import load_config
    from psrl_b200.trainer.strategies import sharded_overlap_mode
    base = ["psrl.fine_grain_overlap.granularity=mini_batch", "psrl.fine_grain_overlap.overlap_scope=pre_step"]
    assert sharded_overlap_mode(load_config(preset="cpu_tiny_grpo", overrides=base)) == "pre_step"
    with pytest.raises(ValueError):
        sharded_overlap_mode(load_config(preset="cpu_tiny_grpo", overrides=base + ["algorithm.use_kl_in_reward=true"]))


def test_gloo_world2_hybrid_multiturn_agentic():
    """Multi-turn sessions (environment observations between turns, version
    pinned at the first turn) through the control-plane process and two
    hybrid ranks."""
    ov = ["psrl.agentic_rl.max_turns=3", "++psrl.agentic_rl.obs_len_min=4", "++psrl.agentic_rl.obs_len_max=8",
          "data.kind=synthetic_tokens", "data.prompt_len_min=8", "data.prompt_len_max=16",
          "data.response_len_mu=1.5", "data.response_len_sigma=0.3", "data.response_len_cap=8",
          "reward.kind=bernoulli_hash", "rollout.ignore_eos=true", "rollout.block_size=4",
          "psrl.staleness_buffer_entries=4", "actor.ppo_mini_batch_size=4"]
    res = _run_sharded(ov)
    assert res[0]["steps"] == [16, 16]


def test_gloo_world2_hybrid_tensor_parallel_rollout():
    """Trainer and rollout engine both at TP=2 over the same two ranks: the
    engine keeps the trainer's shards, the leader feeds both ranks the same
    schedule."""
    res = _run_sharded(["++actor.tensor_parallel_size=2", "++rollout.tensor_parallel_size=2"])
    assert res[0]["steps"] == [32, 32]


def _run_disagg(overrides, world=3):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_disagg_sharded, args=(r, world, port, q, overrides)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(900)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    return q.get(timeout=5)


def test_gloo_world4_disaggregated_tensor_parallel_rollout():
    """Two trainer ranks (data parallel) and one rollout instance of two
    tensor-parallel ranks: the leader takes the work and broadcasts each round,
    both ranks pull the model and keep their shards, and both step in lockstep."""
    res = _run_disagg(["rollout.tensor_parallel_size=2"], world=4)
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world5_disaggregated_heterogeneous_rollout():
    """Rollout instances of different sizes in one job: a TP=2 instance and a
    TP=1 instance serve the same run."""
    res = _run_disagg(["++rollout.tensor_parallel_sizes=[2,1]"], world=5)
    assert res["steps"] == [32, 32] and res["pulls"] >= 3


@pytest.mark.parametrize("trainer", ["++actor.expert_parallel_size=2", "++actor.tensor_parallel_size=2"])
def test_gloo_world4_disaggregated_moe_expert_parallel_rollout(trainer):
    """MoE: an expert-parallel (or expert-tensor-parallel) trainer pair
    publishes its experts; one rollout instance of two ranks splits the
    experts between them (expert parallelism following rollout TP) after
    pulling the full model."""
    res = _run_disagg(["model.preset=tiny-moe", trainer, "rollout.tensor_parallel_size=2"], world=4)
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world3_disaggregated_expert_tensor_parallel_trainer():
    """MoE with trainer TP=2 (every expert split along its width): both ranks
    publish their shards, the rollout rank assembles the full experts while
    it pulls."""
    res = _run_disagg(["model.preset=tiny-moe", "++actor.tensor_parallel_size=2"])
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world4_disaggregated_tp_trainer_and_tp_rollout():
    """The PPO-7B layout in miniature: trainer TP=2 publishing its shards, one
    TP=2 rollout instance pulling them and re-slicing its own shards, PPO with
    a critic."""
    res = _run_disagg(["++actor.tensor_parallel_size=2", "rollout.tensor_parallel_size=2", "critic.enable=true",
                       "algorithm.adv_estimator=gae"], world=4)
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world3_disaggregated_pipeline_parallel_trainer():
    """Two trainer ranks as two pipeline stages, each publishing its own layers;
    the rollout rank pulls every tensor from the stage that holds it."""
    res = _run_disagg(["++actor.pipeline_parallel_size=2"])
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world3_disaggregated_interleaved_pipeline_trainer():
    """Two pipeline ranks with two virtual stages each (four 1-layer chunks,
    interleaved schedule); the rollout rank pulls every tensor from the rank
    that holds it."""
    res = _run_disagg(["++model.overrides.num_layers=4", "++actor.pipeline_parallel_size=2",
                       "++actor.virtual_pipeline_parallel_size=2"])
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


@pytest.mark.parametrize("layout", [[], ["++actor.pipeline_parallel_size=2"]])
def test_gloo_world3_disaggregated_checkpoint_resume(tmp_path, layout):
    """Checkpoints every step (each trainer rank its part, a pipeline stage its
    own layers; rank 0 the data cursor and the marker), then a new run resumes
    at the last step: the PS version and the step counter continue."""
    d = str(tmp_path / "ckpt")
    first = _run_disagg([f"trainer.default_local_dir={d}", "trainer.save_freq=1"] + layout)
    assert first["step_ids"] == [0, 1]
    from psrl_b200.utils.checkpoint import find_latest
    assert find_latest(d) == 2
    again = _run_disagg([f"trainer.default_local_dir={d}", "trainer.resume_mode=auto"] + layout)
    assert again["step_ids"] == [2, 3] and again["steps"] == [32, 32]


def test_gloo_world3_disaggregated_event_logs(tmp_path):
    """trainer.event_log_dir: every rank writes its begin / end spans (trainer
    ranks WAIT / TRAIN / PUSH per step, the rollout rank its PULLs) for the
    timeline viewer; trainer.engine_stats_path: the control plane records the
    instances' engine snapshots."""
    import json
    d = str(tmp_path / "events")
    stats = str(tmp_path / "engine_stats.jsonl")
    res = _run_disagg([f"++trainer.event_log_dir={d}", f"++trainer.engine_stats_path={stats}",
                       "++trainer.engine_stats_interval_s=0.05"])
    assert res["steps"] == [32, 32]
    kinds = {}
    for r in range(3):
        with open(os.path.join(d, f"events_rank{r}.jsonl")) as fh:
            evs = [json.loads(line) for line in fh]
        kinds[r] = {e["type"] for e in evs if e.get("phase") == "end"}
    assert {"WAIT", "TRAIN", "PUSH"} <= kinds[0] and {"WAIT", "TRAIN", "PUSH"} <= kinds[1], kinds
    assert "PULL" in kinds[2], kinds
    from psrl_b200.utils.visualize import main as render_timeline, spans
    with open(os.path.join(d, "events_rank0.jsonl")) as fh:
        assert len(spans([json.loads(line) for line in fh])) >= 6
    html = str(tmp_path / "timeline.html")
    assert render_timeline([d, html]) == 0
    with open(html) as fh:
        page = fh.read()
    assert "trainer0" in page and "rollout2" in page
    # the control plane's engine snapshots of the rollout instance
    from psrl_b200.rollout.stats import StatsRecorder
    recs = StatsRecorder(stats).read()
    assert recs and all(r["instance_id"] == [0, 0] for r in recs)


def test_gloo_world3_disaggregated_validation():
    """trainer.test_freq=1 in the disaggregated placement: after each step the
    rollout instance generates the validation prompts, which are scored and
    never enter a training buffer."""
    res = _run_disagg(["trainer.test_freq=1", "++data.val_size=4"])
    assert res["steps"] == [32, 32]
    assert res["val"] == [4, 4], res


def test_gloo_world3_disaggregated_ulysses_trainer():
    """Two trainer ranks splitting every micro-batch's tokens (Ulysses SP=2)."""
    res = _run_disagg(["++actor.ulysses_sequence_parallel_size=2"])
    assert res["steps"] == [32, 32] and res["pulls"] >= 2


def test_gloo_world3_disaggregated_context_parallel_trainer():
    """Two trainer ranks splitting every sequence (CP=2)."""
    res = _run_disagg(["++actor.context_parallel_size=2"])
    assert res["steps"] == [32, 32] and res["pulls"] >= 2
