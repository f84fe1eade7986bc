"""Host KV offload in the rollout engine (C29): with a KV cache too small for
the batch, preempted sequences' blocks go to the host store and come back on
resume; the greedy tokens equal those of an engine that never preempts, and
resumed sequences recompute fewer tokens than without the store."""

import torch


def _run(num_blocks, offload_blocks):
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    a = PRESETS["tiny"]
    m = build_model(a, "cpu", torch.float32, seed=6)
    eng = RolloutEngine(a, EngineWeights.from_model(m, dtype=torch.float32), max_num_seqs=4, max_model_len=256,
                        block_size=8, num_blocks=num_blocks, max_num_batched_tokens=64, use_cuda_graph=False,
                        enable_prefix_caching=False, kv_offload_blocks=offload_blocks)
    g = torch.Generator().manual_seed(1)
    for i in range(4):
        p = torch.randint(3, a.vocab_size, (30 + 7 * i,), generator=g).tolist()
        eng.add_request(GenRequest(i, p, SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True)))
    outs = {}
    while eng.has_unfinished():
        for o in eng.step():
            outs[o.request_id] = o.output_ids
    return outs, eng.stats


def test_offload_on_preemption_matches_unconstrained_engine():
    ref, st_ref = _run(num_blocks=200, offload_blocks=0)
    assert st_ref["preemptions"] == 0
    plain, st_plain = _run(num_blocks=26, offload_blocks=0)
    off, st_off = _run(num_blocks=26, offload_blocks=128)
    assert st_plain["preemptions"] > 0 and st_off["preemptions"] > 0
    assert st_off["offloaded_blocks"] > 0 and st_off["onloaded_blocks"] > 0
    assert off == ref and plain == ref
    # resumed sequences took their KV from the host instead of re-running prefill
    assert st_off["prefill_tokens"] < st_plain["prefill_tokens"]


def test_offload_on_preemption_gpu():
    """The same on a B200: pinned host blocks moved by the KV block kernel
    over the host link; greedy tokens agree with an engine that never preempts
    (bf16 batch compositions differ, so near-ties may flip)."""
    import pytest
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.rollout import EngineWeights, GenRequest, RolloutEngine, SamplingParams
    a = PRESETS["tiny128"]
    m = build_model(a, "cuda", torch.bfloat16, seed=6)

    def run(num_blocks, off):
        eng = RolloutEngine(a, EngineWeights.from_model(m), max_num_seqs=4, max_model_len=1024, block_size=64,
                            num_blocks=num_blocks, max_num_batched_tokens=512, use_cuda_graph=True,
                            enable_prefix_caching=False, kv_offload_blocks=off)
        g = torch.Generator().manual_seed(1)
        for i in range(4):
            p = torch.randint(3, a.vocab_size, (200 + 90 * i,), generator=g).tolist()
            eng.add_request(GenRequest(i, p, SamplingParams(temperature=0.0, max_tokens=120, ignore_eos=True)))
        outs = {}
        while eng.has_unfinished():
            for o in eng.step():
                outs[o.request_id] = o.output_ids
        return outs, eng.stats

    ref, _ = run(200, 0)
    off, st = run(20, 64)
    assert st["preemptions"] > 0 and st["onloaded_blocks"] > 0
    agree = sum(int(x == y) for i in ref for x, y in zip(ref[i], off[i]))
    total = sum(len(v) for v in ref.values())
    assert agree / total > 0.9, (agree, total)


test_offload_on_preemption_gpu.pytestmark = [__import__("pytest").mark.gpu]
