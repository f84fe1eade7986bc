"""GPU: VMM sleep/wake regions, KV block copies (device <-> pinned host)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_vmm_sleep_wake_backup_and_release():
    from psrl_b200.parallel.memory import MemoryPool
    pool = MemoryPool("cuda:0")
    t = pool.tensor("weights", (1 << 24,), torch.bfloat16)       # 32 MB
    kv = pool.tensor("kv", (1 << 26,), torch.float32)            # 256 MB
    t.copy_(torch.arange(t.numel(), device="cuda").bfloat16())
    kv.fill_(3.0)
    ref = t.clone()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    pool.sleep("kv", backup=False)
    pool.sleep("weights", backup=True)
    free1, _ = torch.cuda.mem_get_info()
    assert free1 - free0 >= (1 << 28)                             # physical memory returned
    assert not pool.is_awake("kv")
    pool.wake("weights")
    pool.wake("kv")
    assert torch.equal(t, ref)                                   # restored from the host copy
    assert float(kv.abs().sum()) == 0.0                          # fresh pages are zero-filled


def test_kv_copy_blocks_device_host_roundtrip():
    from psrl_b200.rollout.kv_offload import copy_blocks
    L, nb, nkv, bs, d = 3, 10, 2, 16, 128
    k = [torch.randn(nb, nkv, bs, d, device="cuda").bfloat16() for _ in range(L)]
    v = [torch.randn(nb, nkv, bs, d, device="cuda").bfloat16() for _ in range(L)]
    hk = [torch.zeros(4, nkv, bs, d, dtype=torch.bfloat16, pin_memory=True) for _ in range(L)]
    hv = [torch.zeros(4, nkv, bs, d, dtype=torch.bfloat16, pin_memory=True) for _ in range(L)]
    copy_blocks(k, v, hk, hv, [7, 2, 5], [0, 1, 3], torch.device("cuda"))
    torch.cuda.synchronize()
    for l in range(L):
        assert torch.equal(hk[l][0], k[l][7].cpu()) and torch.equal(hv[l][3], v[l][5].cpu())
    k2 = [torch.zeros_like(x) for x in k]
    v2 = [torch.zeros_like(x) for x in v]
    copy_blocks(hk, hv, k2, v2, [0, 1, 3], [4, 8, 9], torch.device("cuda"))
    torch.cuda.synchronize()
    for l in range(L):
        assert torch.equal(k2[l][4], k[l][7]) and torch.equal(v2[l][9], v[l][5])


def test_engine_sleep_releases_memory_and_wakes_to_identical_tokens():
    """A rollout engine on a memory pool: sleep releases its KV cache and weights
    (weights kept as a pinned host copy), wake maps them back at the same
    addresses, and the captured decode graphs then produce exactly the greedy
    tokens they produced before the sleep."""
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.memory import MemoryPool
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    a = PRESETS["tiny128"]
    m = build_model(a, "cuda", torch.bfloat16, seed=3)
    pool = MemoryPool("cuda:0")
    eng = RolloutEngine(a, EngineWeights.from_model(m), max_num_seqs=8, max_model_len=512, block_size=64,
                        num_blocks=256, use_cuda_graph=True, memory_pool=pool)
    del m
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, a.vocab_size, (n,), generator=g).tolist() for n in (12, 40, 77)]

    def run(base):
        for i, p in enumerate(prompts):
            eng.add_request(GenRequest(base + i, p, SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)))
        got = {}
        while eng.has_unfinished():
            for o in eng.step():
                got[o.request_id - base] = o.output_ids
        return got

    before = run(0)
    # interrupt one in-flight request with the sleep: it comes back as an abort
    eng.add_request(GenRequest(99, prompts[0], SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)))
    eng.step()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    outs, freed = eng.sleep(keep_weights=True)
    free1, _ = torch.cuda.mem_get_info()
    assert [o.request_id for o in outs] == [99] and outs[0].finish_reason == "abort"
    kv_bytes = sum(t.numel() * t.element_size() for t in eng.k_cache + eng.v_cache)
    assert freed >= kv_bytes and free1 - free0 >= kv_bytes
    eng.wake()
    after = run(100)
    assert after == before


def test_colocated_time_sharing_with_sleep_mode():
    """Colocated trainer + engine alternating (no overlap) with the engine asleep
    during every training phase: steps complete and the engine serves the
    next version after waking."""
    from psrl_b200.config import load_config
    from psrl_b200.trainer import RLTrainer
    cfg = load_config(preset="cpu_tiny_grpo", overrides=[
        "model.preset=tiny128", "model.dtype=bf16", "trainer.device=cuda", "rollout.cuda_graph=true",
        "rollout.enable_sleep_mode=true", "psrl.deployment.colocate_overlap=false",
        "data.kind=synthetic_tokens", "data.prompt_len_min=16", "data.prompt_len_max=64",
        "data.response_len_mu=3.0", "data.response_len_sigma=0.5", "data.response_len_cap=64",
        "reward.kind=bernoulli_hash", "rollout.ignore_eos=true"])
    t = RLTrainer(cfg)
    for _ in range(3):
        m = t.step()
        assert m["num_trajectories"] == 32
        assert not t.engine.asleep
    assert t.engine.version == 3
