"""Layout-transforming weight pull (parallel.weight_sync.ShardedWeightPuller):
trainer stores holding tensor-parallel shards, or pipeline stages' layers, are
copied straight into the rollout engine's full layout; the result equals the
unsharded model's tensors exactly."""

from dataclasses import replace

import pytest
import torch


def _full_layout(a):
    from psrl_b200.trainer.distributed import full_model_layout
    return full_model_layout(a, torch.float32)


def _store(entries_tensors):
    """A CPU store: tensors back to back (64-element aligned) + its entries."""
    entries, off, parts = [], 0, []
    for name, t in entries_tensors:
        entries.append((name, tuple(t.shape), off))
        parts.append((off, t))
        off += (t.numel() + 63) // 64 * 64
    flat = torch.zeros(off)
    for o, t in parts:
        flat[o:o + t.numel()] = t.reshape(-1)
    return {"kind": "shm", "tensor": flat, "entries": entries}


@pytest.mark.parametrize("P,nkv,moe", [(2, 2, False), (4, 2, False), (2, 2, True)])
def test_tensor_parallel_shards_pull_into_full_layout(P, nkv, moe):
    """TP trainer shards (for MoE: every expert, and the shared expert, split
    along its width under the unsharded name) are copied into the full layout."""
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.models.converters import shard_tensor
    from psrl_b200.parallel.assemble import _TP_NAMES
    from psrl_b200.parallel.weight_sync import ShardedWeightPuller
    if moe:
        a = replace(PRESETS["tiny-moe"], num_heads=8, num_kv_heads=nkv, head_dim=16, hidden_size=128,
                    moe_intermediate_size=64, shared_expert_intermediate_size=64)
    else:
        a = replace(PRESETS["tiny"], num_heads=8, num_kv_heads=nkv, head_dim=16, hidden_size=128,
                    intermediate_size=256)
    m = build_model(a, "cpu", torch.float32, seed=1)
    full = dict(m.named_parameters())
    inv = {v: k for k, v in _TP_NAMES.items()}
    stores = []
    for r in range(P):
        items = []
        for n, t in full.items():
            suffix = next((k for k in inv if n.endswith(k)), None)
            if suffix is not None:                       # sharded: the TP trainer's local name
                items.append((n[: -len(suffix)] + inv[suffix], shard_tensor(t.detach(), n, a, r, P)))
            elif "experts_w" in n or "shared_gate_up" in n or "shared_down" in n:
                items.append((n, shard_tensor(t.detach(), n, a, r, P)))   # expert TP: same name
            else:
                items.append((n, t.detach()))
        d = _store(items)
        d.update(tp_rank=r, tp_world=P)
        stores.append(d)
    lay = _full_layout(a)
    dst = torch.full((lay.total,), float("nan"))
    ShardedWeightPuller(lay, stores, dst, a).pull()
    views = lay.views(dst)
    for n, t in full.items():
        torch.testing.assert_close(views[n], t.detach(), rtol=0, atol=0)


def test_pipeline_stage_stores_pull_into_full_layout():
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.weight_sync import ShardedWeightPuller
    a = replace(PRESETS["tiny"], num_layers=4)
    m = build_model(a, "cpu", torch.float32, seed=2)
    full = dict(m.named_parameters())
    stage_of = lambda n: 0 if n.startswith("embed") else (1 if not n.startswith("layers.") else
                                                            int(n.split(".")[1]) // 2)
    stores = [_store([(n, t.detach()) for n, t in full.items() if stage_of(n) == s]) for s in range(2)]
    stores.append(_store([(n, t.detach()) for n, t in full.items() if stage_of(n) == 1]))   # a DP replica
    lay = _full_layout(a)
    dst = torch.full((lay.total,), float("nan"))
    p = ShardedWeightPuller(lay, stores, dst, a)
    p.pull()
    views = lay.views(dst)
    for n, t in full.items():
        torch.testing.assert_close(views[n], t.detach(), rtol=0, atol=0)
    assert {j for j, *_ in p.blocks} == {0, 1, 2}        # stage 1's tensors spread over both replicas


@pytest.mark.gpu
def test_tensor_parallel_pull_kernel_gpu():
    """The same plan through the copy_rows kernel on a B200 (stores in device
    memory of this process: the kernel's loads are the ones it makes from a
    peer's HBM)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.models.converters import shard_tensor
    from psrl_b200.parallel.assemble import _TP_NAMES
    from psrl_b200.parallel.weight_sync import ShardedWeightPuller
    from psrl_b200.trainer.distributed import full_model_layout
    a = PRESETS["qwen2.5-3b"]
    a = replace(a, num_layers=2)
    m = build_model(a, "cuda", torch.bfloat16, seed=1)
    full = dict(m.named_parameters())
    inv = {v: k for k, v in _TP_NAMES.items()}
    stores = []
    for r in range(2):
        items = []
        for n, t in full.items():
            suffix = next((k for k in inv if n.endswith(k)), None)
            items.append((n[: -len(suffix)] + inv[suffix], shard_tensor(t.detach(), n, a, r, 2)) if suffix else
                         (n, t.detach()))
        d = _store([(n, t.float().cpu()) for n, t in items])
        d["tensor"] = d["tensor"].to("cuda", torch.bfloat16)
        d.update(tp_rank=r, tp_world=2)
        stores.append(d)
    lay = full_model_layout(a, torch.bfloat16)
    dst = torch.zeros(lay.total, dtype=torch.bfloat16, device="cuda")
    p = ShardedWeightPuller(lay, stores, dst, a)
    n = p.pull()
    torch.cuda.synchronize()
    views = lay.views(dst)
    for name, t in full.items():
        torch.testing.assert_close(views[name], t.detach(), rtol=0, atol=0)
    assert n >= sum(t.numel() * 2 for t in full.values())


@pytest.mark.parametrize("preset,P", [("tiny", 2), ("tiny", 4), ("tiny-moe", 2)])
def test_engine_shard_pull_from_whole_tensor_stores(preset, P):
    """A TP rollout rank's direct shard pull from data-parallel trainer stores
    equals slicing the full model (shard_engine_tensors), for every rank, also
    with more ranks than KV heads and with experts split by expert."""
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.parallel.tp import TPGroup, shard_engine_tensors
    from psrl_b200.parallel.weight_sync import EngineShardPuller
    a = PRESETS[preset]
    m = build_model(a, "cpu", torch.float32, seed=3)
    full = {n: p.detach() for n, p in m.named_parameters()}
    lay = _full_layout(a)
    flat = torch.zeros(lay.total)
    views = lay.views(flat)
    for n, t in full.items():
        views[n].copy_(t)
    stores = [{"kind": "shm", "tensor": flat}, {"kind": "shm", "tensor": flat.clone()}]
    for r in range(P):
        pl = EngineShardPuller(lay, stores, a, r, P)
        pl.pull()
        want = shard_engine_tensors(a, full, TPGroup(None, P, r))
        for n, t in want.items():
            torch.testing.assert_close(pl.tensors[n], t, rtol=0, atol=0)


def test_engine_shard_pull_from_same_size_tp_stores():
    """Trainer TP=2 stores (local names, own shards) feed a TP=2 engine rank
    directly: rank r copies trainer rank r's shards whole."""
    from psrl_b200.models import PRESETS, build_model
    from psrl_b200.models.converters import shard_tensor
    from psrl_b200.parallel.assemble import _TP_NAMES
    from psrl_b200.parallel.tp import TPGroup, shard_engine_tensors
    from psrl_b200.parallel.weight_sync import EngineShardPuller
    a = PRESETS["tiny"]
    P = 2
    full = {n: p.detach() for n, p in build_model(a, "cpu", torch.float32, seed=4).named_parameters()}
    inv = {v: k for k, v in _TP_NAMES.items()}
    stores = []
    for r in range(P):
        items = []
        for n, t in full.items():
            suffix = next((k for k in inv if n.endswith(k)), None)
            items.append((n[: -len(suffix)] + inv[suffix], shard_tensor(t, n, a, r, P)) if suffix else (n, t))
        d = _store(items)
        d.update(tp_rank=r, tp_world=P)
        stores.append(d)
    lay = _full_layout(a)
    for r in range(P):
        pl = EngineShardPuller(lay, stores, a, r, P)
        pl.pull()
        for n, t in shard_engine_tensors(a, full, TPGroup(None, P, r)).items():
            torch.testing.assert_close(pl.tensors[n], t, rtol=0, atol=0)
