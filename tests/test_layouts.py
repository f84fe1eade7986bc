"""Comm planning (finest shard mesh, balancing, merging) and TP layouts."""

import pytest
import torch

from psrl_b200.models import PRESETS, build_model
from psrl_b200.models.converters import copy_segments_for, local_shape, shard_tensor, tp_slices
from psrl_b200.parallel.comm_plan import NetworkTopology, Sharding, TensorSpec, merge_contiguous, plan_transfer, Segment


def _apply(plan, spec, sender_bufs, dst):
    flat = dst.view(-1).view(torch.uint8)
    for s in plan.segments:
        src = sender_bufs[s.src].view(-1).view(torch.uint8)
        flat[s.dst_off: s.dst_off + s.nbytes] = src[s.src_off: s.src_off + s.nbytes]


def test_plan_fsdp4_to_tp2_rows():
    full = torch.arange(16 * 6, dtype=torch.float32).view(16, 6)
    spec = TensorSpec("w", (16, 6), 4)
    senders = {i: {"w": Sharding(0, 4, i)} for i in range(4)}
    bufs = {i: full[i * 4:(i + 1) * 4].contiguous() for i in range(4)}
    for r in range(2):
        plan = plan_transfer([spec], senders, {"w": Sharding(0, 2, r)})
        dst = torch.zeros(8, 6)
        _apply(plan, spec, bufs, dst)
        assert torch.equal(dst, full[r * 8:(r + 1) * 8])
        assert len(plan.segments) == 2          # one merged run per sender


def test_plan_balances_replicated_senders():
    spec = TensorSpec("w", (12, 4), 2)
    senders = {i: {"w": Sharding(0, 1, 0)} for i in range(3)}   # full replicas
    plan = plan_transfer([spec], senders, {"w": Sharding(0, 3, 1)})
    assert plan.total_bytes() == 4 * 4 * 2
    plan_all = plan_transfer([spec], senders, {"w": Sharding(0, 1, 0)})
    # lcm(1,1)=1 piece -> one sender; with a 3-way receiver split pieces spread
    assert plan_all.total_bytes() == 12 * 4 * 2
    assert NetworkTopology({0: 0, 1: 1}).link(0, 1) == "ib"


def test_merge_contiguous():
    segs = [Segment("a", 0, 0, 0, 8), Segment("a", 0, 8, 8, 8), Segment("a", 1, 16, 16, 8)]
    assert len(merge_contiguous(segs)) == 2


@pytest.mark.parametrize("preset", ["tiny128", "tiny-moe-shared"])
def test_tp_slices_reconstruct_and_segments(preset):
    from dataclasses import replace
    a = PRESETS[preset] if preset != "tiny-moe-shared" else replace(PRESETS["tiny-moe"],
                                                                     shared_expert_intermediate_size=128)
    m = build_model(a, "cpu", torch.float32)
    for name, p in m.named_parameters():
        t = 2
        parts = [shard_tensor(p.data, name, a, r, t) for r in range(t)]
        for r in range(t):
            assert tuple(parts[r].shape) == local_shape(name, tuple(p.shape), a, r, t)
            # byte runs reproduce the same local tensor
            dst = torch.zeros(parts[r].numel())
            srcb = p.data.contiguous().view(-1).view(torch.uint8)
            dstb = dst.view(torch.uint8)
            for so, do, nb in copy_segments_for(name, tuple(p.shape), 4, a, r, t, 0, 0):
                dstb[do:do + nb] = srcb[so:so + nb]
            assert torch.equal(dst.view(parts[r].shape), parts[r]), name
    qkv = tp_slices("layers.0.attn.qkv.weight", (a.qkv_size, a.hidden_size), a, 1, 2)
    assert qkv[0] == (0, 4 * 128, 4 * 128)
