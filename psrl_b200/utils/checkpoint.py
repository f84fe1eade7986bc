"""Checkpoint / resume (reference: ``ray_trainer.py:2413-2560``, C36).

Layout under ``trainer.default_local_dir``::

    global_step_{N}/actor/config.json, model*.safetensors   (HF format, rank 0)
    global_step_{N}/actor/dcp/                             (torch DCP, when use_dcp_save)
    global_step_{N}/actor/optim_rank{r}.pt                  (per-rank optimizer shard)
    global_step_{N}/critic/...                              (same, if a critic exists)
    global_step_{N}/data.pt                                 (data cursor, PS version)
    latest_checkpointed_iteration.txt

The optimizer state is saved per rank (the reference's per-rank Megatron save
avoids DCP's collective object gathers); model weights are saved in HF format
and, optionally, as a torch Distributed Checkpoint.  Resuming at step N sets the
PS version to N (the version after N trainer steps).
"""

from __future__ import annotations

import os

import torch

from ..models.hf_io import load_hf_into, save_hf

LATEST = "latest_checkpointed_iteration.txt"


def step_dir(root: str, step: int) -> str:
    return os.path.join(os.path.expanduser(root), f"global_step_{step}")


def _is_sharded(worker) -> bool:
    return getattr(worker, "tp", None) is not None or getattr(worker, "ep", None) is not None


def _full_model_from_shards(worker):
    """The unsharded model (CPU, fp32) assembled from a TP / EP worker's shards;
    a collective over the worker's TP / EP groups (every rank calls it)."""
    from ..models.qwen import QwenModel
    from ..parallel.assemble import FullWeightAssembler
    m = worker.model
    asm = FullWeightAssembler(
        m, ep=worker.ep, tp=worker.tp,
        ep_names=[n for n, _ in m.named_parameters() if "experts_w" in n] if worker.ep is not None else (),
        tp_names=sorted(worker.tp_sharded) if worker.tp is not None else ())
    full = QwenModel(worker.args)
    asm.gather()
    tensors = {n: p.data for n, p in full.named_parameters()}
    asm.assemble_into(tensors)
    return full


def _shard_into(worker, full) -> None:
    """Copy this rank's shards of an unsharded model into a TP / EP worker."""
    fp = {n: p.detach() for n, p in full.named_parameters()}
    with torch.no_grad():
        for n, p in worker.model.named_parameters():
            if worker.tp is not None:
                # the trainer's TP layout (``models.converters.tp_slices``): heads,
                # MLP width and, for MoE, every expert's width
                from ..models.converters import shard_tensor
                from ..parallel.assemble import engine_name
                en = engine_name(n)
                src = fp[en]
                if n in worker.tp_sharded:
                    src = shard_tensor(src, en, worker.args, worker.tp.rank, worker.tp.world)
            else:
                src = fp[n]
            if worker.ep is not None and "experts_w" in n:
                src = src[worker.ep.first: worker.ep.first + worker.ep.local]
            p.copy_(src.to(p.dtype))


def save_worker(worker, path: str, rank: int = 0, use_dcp: bool = False, group=None) -> None:
    """``group``: the process group of the ranks that save together (DCP's
    coordination; default: every rank of the job)."""
    os.makedirs(path, exist_ok=True)
    if getattr(worker, "pp", None) is not None:
        # a pipeline stage holds only its layers: every rank keeps its own file
        torch.save({k: v.detach().cpu() for k, v in worker.model.state_dict().items()},
                   os.path.join(path, f"model_rank{rank}.pt"))
    elif _is_sharded(worker):
        # HF export of the whole model, assembled from the TP / EP shards (collective)
        full = _full_model_from_shards(worker)
        if rank == 0:
            save_hf(full, path)
        partner = getattr(worker, "dp_partner", None)
        if partner is not None:
            torch.save(partner.optimizer_state(), os.path.join(path, f"optim_partner_rank{rank}.pt"))
    elif rank == 0:
        save_hf(worker.model, path)
    if use_dcp:
        import torch.distributed.checkpoint as dcp
        sd = {k: v.detach() for k, v in worker.model.state_dict().items()}
        dcp.save(sd, checkpoint_id=os.path.join(path, "dcp"), process_group=group)
    if worker.dp is not None:
        torch.save(worker.dp.optimizer_state(), os.path.join(path, f"optim_rank{rank}.pt"))


def load_worker(worker, path: str, rank: int = 0, use_dcp: bool = False, group=None) -> None:
    stage_file = os.path.join(path, f"model_rank{rank}.pt")
    if getattr(worker, "pp", None) is not None:
        sd = torch.load(stage_file, map_location="cpu", weights_only=False)
        with torch.no_grad():
            for k, v in worker.model.state_dict().items():
                v.copy_(sd[k].to(v.dtype))
    elif use_dcp and os.path.isdir(os.path.join(path, "dcp")):
        import torch.distributed.checkpoint as dcp
        sd = {k: v.detach() for k, v in worker.model.state_dict().items()}
        dcp.load(sd, checkpoint_id=os.path.join(path, "dcp"), process_group=group)
    elif _is_sharded(worker):
        from ..models.qwen import QwenModel
        full = QwenModel(worker.args)
        load_hf_into(full, path)
        _shard_into(worker, full)
    else:
        load_hf_into(worker.model, path)
    opt = os.path.join(path, f"optim_rank{rank}.pt")
    if worker.dp is not None:
        if os.path.exists(opt):
            worker.dp.load_optimizer_state(torch.load(opt, map_location="cpu", weights_only=False))
        else:
            worker.dp.sync_master_from_params()
    partner = getattr(worker, "dp_partner", None)
    if partner is not None:
        popt = os.path.join(path, f"optim_partner_rank{rank}.pt")
        if os.path.exists(popt):
            partner.load_optimizer_state(torch.load(popt, map_location="cpu", weights_only=False))
        else:
            partner.sync_master_from_params()


def save_checkpoint(root: str, step: int, actor, data=None, critic=None, ps_version: int | None = None,
                    rank: int = 0, use_dcp: bool = False, extra: dict | None = None) -> str:
    """``extra``: small trainer state kept beside the data cursor (e.g. the
    adaptive in-reward KL coefficient); :func:`load_checkpoint` returns it
    through ``extra_out``."""
    d = step_dir(root, step)
    save_worker(actor, os.path.join(d, "actor"), rank, use_dcp)
    if critic is not None:
        save_worker(critic, os.path.join(d, "critic"), rank, use_dcp)
    if rank == 0:
        torch.save({"data": data.state_dict() if data is not None else None, "ps_version": ps_version,
                    "global_step": step, "extra": dict(extra or {})}, os.path.join(d, "data.pt"))
        with open(os.path.join(os.path.expanduser(root), LATEST), "w") as fh:
            fh.write(str(step))
    return d


def find_latest(root: str) -> int | None:
    p = os.path.join(os.path.expanduser(root), LATEST)
    if not os.path.exists(p):
        return None
    with open(p) as fh:
        return int(fh.read().strip())


def load_checkpoint(root: str, actor, data=None, critic=None, step: int | None = None, rank: int = 0,
                    use_dcp: bool = False, extra_out: dict | None = None) -> int:
    step = find_latest(root) if step is None else step
    if step is None:
        raise FileNotFoundError(f"no checkpoint under {root}")
    d = step_dir(root, step)
    load_worker(actor, os.path.join(d, "actor"), rank, use_dcp)
    if critic is not None:
        load_worker(critic, os.path.join(d, "critic"), rank, use_dcp)
    meta = torch.load(os.path.join(d, "data.pt"), weights_only=False)
    if data is not None and meta.get("data"):
        data.load_state_dict(meta["data"])
    if extra_out is not None:
        extra_out.update(meta.get("extra") or {})
    return int(meta["global_step"])


# --------------------------------------------------- multi-GPU placements
def save_trainer_ranks(root: str, step: int, actor, critic, rank: int, meta: dict | None, use_dcp: bool = False,
                       extra: dict | None = None, group=None) -> str:
    """Every trainer rank of a multi-GPU placement calls this (the HF export of
    TP / EP shards is collective); rank 0 also writes ``data.pt`` from
    ``meta`` (the control plane's data cursor and PS version) and, last, the
    latest-step marker, so a half-written step is never the one resumed."""
    d = step_dir(root, step)
    save_worker(actor, os.path.join(d, "actor"), rank, use_dcp, group)
    if critic is not None:
        save_worker(critic, os.path.join(d, "critic"), rank, use_dcp, group)
    return d


def finish_trainer_checkpoint(root: str, step: int, meta: dict | None, extra: dict | None = None) -> None:
    """Rank 0, after every trainer rank saved its part (a barrier in between)."""
    d = step_dir(root, step)
    torch.save({"data": (meta or {}).get("data"), "ps_version": (meta or {}).get("ps_version"),
                "global_step": step, "extra": dict(extra or {})}, os.path.join(d, "data.pt"))
    with open(os.path.join(os.path.expanduser(root), LATEST), "w") as fh:
        fh.write(str(step))


def load_trainer_ranks(root: str, step: int, actor, critic, rank: int, use_dcp: bool = False, group=None) -> dict:
    """Every trainer rank loads its part of step ``step``; returns the extra
    trainer state saved beside the data cursor."""
    d = step_dir(root, step)
    load_worker(actor, os.path.join(d, "actor"), rank, use_dcp, group)
    if critic is not None:
        load_worker(critic, os.path.join(d, "critic"), rank, use_dcp, group)
    meta = torch.load(os.path.join(d, "data.pt"), weights_only=False)
    return dict(meta.get("extra") or {})
