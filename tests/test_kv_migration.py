"""Migration of a running request between two rollout engines together with
its KV blocks: the destination continues with a one-token prefill and the
greedy output equals an unmigrated run.  CPU (fp32, same process) and two
B200s (KV blocks read over NVLink by the block kernel)."""

import pytest
import torch


def _engine(a, m, device, dtype):
    from psrl_b200.rollout import EngineWeights, RolloutEngine
    return RolloutEngine(a, EngineWeights.from_model(m, device=device, dtype=dtype), max_num_seqs=4,
                         max_model_len=512, block_size=16 if device == "cpu" else 64, num_blocks=64,
                         max_num_batched_tokens=256, use_cuda_graph=device != "cpu", enable_prefix_caching=False)


def _prompts(a):
    g = torch.Generator().manual_seed(3)
    return [torch.randint(3, a.vocab_size, (n,), generator=g).tolist() for n in (37, 90, 21)]


def _run(src, dst, prompts, migrate_after: int | None):
    from psrl_b200.rollout import GenRequest, SamplingParams
    for i, p in enumerate(prompts):
        src.add_request(GenRequest(i, p, SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True)))
    outs, steps, moved = {}, 0, False
    while src.has_unfinished() or (dst is not None and dst.has_unfinished()):
        if src.has_unfinished():
            for o in src.step():
                outs[o.request_id] = o.output_ids
        if dst is not None and dst.has_unfinished():
            for o in dst.step():
                outs[o.request_id] = o.output_ids
        steps += 1
        if migrate_after is not None and steps == migrate_after and not moved:
            moved = src.migrate_request(1, dst)
    return outs, moved


def test_migrate_with_kv_cpu():
    from psrl_b200.models import PRESETS, build_model
    a = PRESETS["tiny"]
    m = build_model(a, "cpu", torch.float32, seed=2)
    prompts = _prompts(a)
    ref, _ = _run(_engine(a, m, "cpu", torch.float32), None, prompts, None)
    src, dst = _engine(a, m, "cpu", torch.float32), _engine(a, m, "cpu", torch.float32)
    got, moved = _run(src, dst, prompts, migrate_after=8)
    assert moved and src.stats["migrated_out"] == 1 and dst.stats["migrated_in"] == 1
    assert got == ref
    assert dst.stats["prefill_tokens"] == 1          # one token recomputed, not the context


@pytest.mark.gpu
def test_migrate_with_kv_across_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from psrl_b200.models import PRESETS, build_model
    a = PRESETS["tiny128"]
    m = build_model(a, "cuda:0", torch.bfloat16, seed=2)
    prompts = _prompts(a)
    ref, _ = _run(_engine(a, m, "cuda:0", torch.bfloat16), None, prompts, None)
    src, dst = _engine(a, m, "cuda:0", torch.bfloat16), _engine(a, m, "cuda:1", torch.bfloat16)
    got, moved = _run(src, dst, prompts, migrate_after=8)
    assert moved and dst.stats["prefill_tokens"] == 1
    agree = sum(int(x == y) for i in ref for x, y in zip(ref[i], got[i]))
    total = sum(len(v) for v in ref.values())
    assert agree / total > 0.9, (agree, total)
