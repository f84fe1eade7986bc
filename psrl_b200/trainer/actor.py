"""Actor / reference / critic workers (the trainer side of the engine, C11).

``PolicyWorker`` owns a decoder in bf16 (fp32 on CPU), the sharded DP optimizer
(:class:`~psrl_b200.parallel.fsdp.FlatShardedDP`) and implements:

* ``compute_log_prob`` — old (or reference) log-probs over packed micro-batches;
* ``update_policy`` — mini-batch / micro-batch PPO-family update with the fused
  LM-head log-prob (K8), clip-higher + dual-clip, token-mean aggregation over
  the global token count, optional entropy bonus, KL loss and TIS weights;
* ``publish_state`` — the parameters to hand to the weight-sync path.

Reference: ``PSRL_EngineTrainWorker`` (``psrl/workers/train/engine_train_worker.py:75``,
``update_actor`` :521) on top of veRL's actor.
"""

from __future__ import annotations

import time

import torch

from ..parallel.cp import CPShard
from ..models import ModelArgs, build_model
from ..parallel.fsdp import FlatShardedDP
from . import algos
from .batch import Trajectory, balance_across_ranks, build_micro_batch, pack_micro_batches, response_slices


def _dtype(name: str, device) -> torch.dtype:
    if torch.device(device).type == "cpu" and name == "bf16":
        return torch.float32
    return {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}[name]


def dist_world(group) -> int:
    import torch.distributed as dist
    return dist.get_world_size(group) if dist.is_initialized() else 1


def mini_batch_groups(trajs: list[Trajectory], mini_batch_size: int) -> list[list[int]]:
    """Split by prompt group into ``mini_batch_size`` groups per mini-batch."""
    by_uid: dict = {}
    for i, t in enumerate(trajs):
        by_uid.setdefault(t.uid, []).append(i)
    groups = list(by_uid.values())
    per = max(1, int(mini_batch_size))
    return [[i for g in groups[s: s + per] for i in g] for s in range(0, len(groups), per)]


def loss_tokens(t: Trajectory) -> int:
    """Response tokens that enter the policy loss (environment tokens of a
    multi-turn response and rejected tokens are masked out)."""
    return int(sum(t.response_mask)) if t.response_mask is not None else t.response_len


def plan_update(trajs: list[Trajectory], mini_batch_size: int, dp_world: int) -> list[list[tuple]]:
    """Per data-parallel rank, the list of ``(my_indices, global_tokens, num_seqs)``
    of every PPO mini-batch (token-balanced split of each mini-batch).  Every
    rank gets one entry per mini-batch, so all ranks take the same number of
    optimizer steps (and collectives)."""
    plans: list[list[tuple]] = [[] for _ in range(dp_world)]
    for mini in mini_batch_groups(trajs, mini_batch_size):
        gt = float(sum(loss_tokens(trajs[i]) for i in mini))
        parts = balance_across_ranks([trajs[i] for i in mini], dp_world)
        for r in range(dp_world):
            plans[r].append(([mini[j] for j in parts[r]], gt, len(mini)))
    return plans


class PolicyWorker:
    def __init__(self, cfg, args: ModelArgs, device, dp_group=None, seed: int = 0, trainable: bool = True,
                 dp_rank: int = 0, dp_world: int = 1, tp_group=None, cp_group=None, pp_group=None,
                 cp_mode: str = "zigzag"):
        self.cfg = cfg
        self.args = args
        self.device = torch.device(device)
        self.dtype = _dtype(cfg.model.dtype, device)
        self.model = build_model(args, self.device, self.dtype, seed=seed)
        self.model.gradient_checkpointing = bool(cfg.model.enable_gradient_checkpointing)
        self.dp_rank, self.dp_world = dp_rank, dp_world
        self.dp = None
        self.dp_partner = None
        self.ep = None
        expert_names: set = set()
        self.tp = None
        # context parallelism: the ranks of cp_group share each micro-batch along
        # the sequence (dp_rank / dp_world index the CP groups; dp_group spans
        # every rank, so gradients sum over data and context parallelism)
        self.cp_group = cp_group if cp_group is not None and dist_world(cp_group) > 1 else None
        # "zigzag": context parallelism (keys / values all-gathered); "ulysses":
        # contiguous token slices, head-parallel attention between two all-to-alls
        if cp_mode not in ("zigzag", "ulysses"):
            raise ValueError(f"unknown sequence-parallel mode {cp_mode!r}")
        self.cp_mode = cp_mode
        # pipeline parallelism: this rank runs one stage of the layers (dp_group
        # then joins the same stage of every pipeline; the clip norm spans the stages)
        self.pp = None
        if pp_group is not None and dist_world(pp_group) > 1:
            if (tp_group is not None and dist_world(tp_group) > 1) or self.cp_group is not None or args.is_moe:
                raise ValueError("pipeline parallelism here combines with data parallelism only")
            from ..parallel.pp import PipelineStage
            meg = cfg.actor.get("megatron", None) or {}
            vpp = max(int(cfg.actor.get("virtual_pipeline_parallel_size", 1) or 1),
                      int(meg.get("virtual_pipeline_model_parallel_size", 1) or 1))
            self.pp = PipelineStage(self.model, pp_group, virtual=vpp)
        if self.cp_group is not None:
            if tp_group is not None and dist_world(tp_group) > 1:
                raise ValueError("context parallelism together with tensor parallelism is not implemented")
            modes = {cfg.actor.loss_agg_mode} | ({cfg.critic.get("loss_agg_mode", "token-mean")}
                                                  if args.value_head else set())
            if not modes <= {"token-mean", "seq-mean-token-sum"}:
                raise ValueError("context parallelism needs a loss that is a sum over tokens "
                                 "(loss_agg_mode token-mean or seq-mean-token-sum)")
        if tp_group is not None and dist_world(tp_group) > 1:
            # tensor parallelism inside tp_group (data parallelism across dp_group)
            from ..parallel.tp import apply_tensor_parallel, make_tp_group
            fused = 0
            if bool(cfg.actor.get("tp_fused_collectives", True)):
                # accumulators for the widest fused all-reduce: one micro-batch x hidden
                rows = max(int(cfg.actor.get("ppo_max_token_len_per_gpu", 10240)),
                           int(cfg.rollout.max_prompt_length) + int(cfg.rollout.max_response_length))
                fused = rows * args.hidden_size
            self.tp = make_tp_group(tp_group, device, fused)
            self.tp_sharded = set(apply_tensor_parallel(self.model, self.tp))
        ep_size = int(cfg.actor.get("expert_parallel_size", 1) or 1)
        if args.is_moe and ep_size > 1 and self.tp is not None:
            raise ValueError("tensor parallelism splits each expert's width (ETP); combining it with expert "
                             "parallelism is not implemented")
        if args.is_moe and ep_size > 1:
            # expert parallelism over the data-parallel group: rank r keeps
            # experts [r E/P, (r+1) E/P) of every layer (K12)
            from ..parallel.ep import make_ep_group, shard_experts
            if dp_group is None or dp_world != ep_size:
                raise ValueError("expert_parallel_size must equal the data-parallel world size")
            p2p_bytes = 0
            if bool(cfg.actor.get("ep_peer_all_to_all", True)):
                # receive buffers for twice a micro-batch's routed rows (rows beyond go through NCCL)
                p2p_bytes = 2 * int(cfg.actor.ppo_max_token_len_per_gpu) * args.num_experts_per_tok * \
                    args.hidden_size * torch.finfo(self.dtype).bits // 8
            self.ep = make_ep_group(dp_group, args.num_experts, device=self.device, p2p_bytes=p2p_bytes)
            expert_names = set(shard_experts(self.model, self.ep))
        if trainable:
            oc = cfg.actor.optim if not args.value_head else cfg.critic.optim
            kw = dict(lr=float(oc.lr), betas=tuple(oc.get("betas", (0.9, 0.999))), eps=float(oc.get("eps", 1e-8)),
                      weight_decay=float(oc.weight_decay), max_grad_norm=float(cfg.actor.grad_clip),
                      warmup_steps=int(oc.get("lr_warmup_steps", 0)))
            if self.tp is not None:
                # TP-sharded parameters: disjoint across the TP group (norm summed over it);
                # replicated parameters: identical across it (counted once)
                sh = self.tp_sharded
                self.dp = FlatShardedDP(self.model, dp_group, param_filter=lambda n: n not in sh, **kw)
                self.dp_partner = FlatShardedDP(self.model, dp_group, param_filter=lambda n: n in sh,
                                                norm_group=tp_group, **kw)
            elif self.pp is not None:
                if self.pp.last and not self.pp.first and args.tie_word_embeddings:
                    # the tied embedding's other copy lives on the first stage, which counts it
                    # in the clip norm; this copy is reduced and updated the same way
                    self.dp = FlatShardedDP(self.model, dp_group, norm_group=pp_group,
                                            param_filter=lambda n: n != "embed.weight", **kw)
                    self.dp_partner = FlatShardedDP(self.model, dp_group, count_in_norm=False,
                                                    param_filter=lambda n: n == "embed.weight", **kw)
                else:
                    self.dp = FlatShardedDP(self.model, dp_group, norm_group=pp_group, **kw)
            else:
                # hybrid sharding: optimizer state sharded over groups of fsdp_size ranks,
                # replicated across them (veRL's fsdp_config.fsdp_size; -1: shard over all)
                fc = cfg.actor.get("fsdp_config", None) or {}
                fsdp_size = int(cfg.actor.get("fsdp_size", -1) or -1)
                fsdp_size = fsdp_size if fsdp_size > 0 else int(fc.get("fsdp_size", -1) or -1)
                shard_group, rep_group = dp_group, None
                if fsdp_size > 0 and dp_group is not None and dist_world(dp_group) > fsdp_size:
                    from ..parallel.fsdp import hybrid_shard_groups
                    shard_group, rep_group = hybrid_shard_groups(dp_group, fsdp_size)
                # gradient sharding: no model-wide fp32 main-grad buffer (large models)
                self.dp = FlatShardedDP(self.model, shard_group, param_filter=lambda n: n not in expert_names,
                                        replicate_group=rep_group,
                                        shard_grads=bool(cfg.actor.get("fsdp_shard_grads", False)), **kw)
            if self.tp is None and expert_names:
                # each rank's experts are its own: no reduction, but the clip norm spans all ranks
                self.dp_partner = FlatShardedDP(self.model, None, param_filter=lambda n: n in expert_names,
                                                norm_group=dp_group, **kw)
            elif self.tp is None and self.pp is None and bool(cfg.actor.get("fsdp_peer_step", True)):
                # fused peer-memory reduce-scatter + AdamW + all-gather (CUDA, world > 1)
                self.dp.enable_peer_step()
        else:
            for p in self.model.parameters():
                p.requires_grad_(False)
        self.max_tokens = int(cfg.actor.ppo_max_token_len_per_gpu)

    # ---------------------------------------------------------------- utils
    def my_share(self, trajs: list[Trajectory], idx: list[int] | None = None) -> list[int]:
        idx = list(range(len(trajs))) if idx is None else idx
        parts = balance_across_ranks([trajs[i] for i in idx], self.dp_world)
        return [idx[j] for j in parts[self.dp_rank]]

    def _lockstep(self, bins: list) -> list:
        """Expert-parallel forwards are collectives over the expert group
        (token dispatch and combine, and their transposes in backward), so
        every rank runs the same number of micro-batches: this rank's list is
        padded with ``None`` up to the group maximum (one all-reduce of an
        int).  A ``None`` entry runs a one-token placeholder whose result is
        discarded (its loss is multiplied by zero).  Gradient sharding needs
        the same: every micro-batch's backward reduce-scatters each layer's
        gradients over the shard group."""
        if self.ep is not None:
            grp = self.ep.group
        elif self.dp is not None and getattr(self.dp, "shard_grads", False):
            grp = self.dp.group
        else:
            return list(bins)
        import torch.distributed as dist
        dev = self.device if self.device.type == "cuda" else torch.device("cpu")
        n = torch.tensor([len(bins)], dtype=torch.int64, device=dev)
        dist.all_reduce(n, op=dist.ReduceOp.MAX, group=grp)
        return list(bins) + [None] * (int(n.item()) - len(bins))

    def _recount_plan(self, trajs: list[Trajectory], plan: list[tuple]) -> list[tuple]:
        """A plan made before rejection sampling counted tokens that are now
        masked: recount each mini-batch's loss tokens over the data-parallel
        group (one all-reduce of one number per mini-batch)."""
        import torch.distributed as dist
        local = torch.tensor([float(sum(loss_tokens(trajs[i]) for i in mine)) for mine, _, _ in plan],
                             dtype=torch.float64)
        grp = self.dp.group if self.dp is not None else None
        if grp is not None and dist.is_initialized() and dist_world(grp) > 1:
            dev = self.device if self.device.type == "cuda" else torch.device("cpu")
            local = local.to(dev)
            dist.all_reduce(local, group=grp)
            local = local.cpu()
        return [(mine, max(1.0, float(n)), ns) for (mine, _, ns), n in zip(plan, local.tolist())]

    def _new_shard(self, cu_seqlens):
        if self.cp_mode == "ulysses":
            from ..parallel.ulysses import UlyssesShard
            return UlyssesShard(cu_seqlens, self.cp_group)
        return CPShard(cu_seqlens, self.cp_group)

    def _cp_shard(self, mb):
        """Under context parallelism, replace ``mb``'s per-token tensors in place
        by this rank's share (``cu_seqlens`` becomes the :class:`CPPlan`) and
        return the function that cuts other per-token tensors the same way;
        otherwise leave ``mb`` alone and return the identity."""
        if self.cp_group is None:
            return lambda t: t
        sh = self._new_shard(mb.cu_seqlens)
        mb.input_ids = sh.local(mb.input_ids)
        mb.labels = sh.local(mb.labels)
        mb.loss_mask = sh.local(mb.loss_mask, 0.0)
        mb.old_logprobs = sh.local(mb.old_logprobs, 0.0)
        mb.advantages = sh.local(mb.advantages, 0.0)
        mb.seq_ids = sh.local(mb.seq_ids)
        if "is_weights" in mb.extra:
            mb.extra["is_weights"] = sh.local(mb.extra["is_weights"], 1.0)
        mb.positions = sh.positions()
        mb.cu_seqlens, mb.max_seqlen = sh.plan, sh.plan.max_q
        return sh.local

    def _main_grad(self, p):
        """The fp32 main-gradient view of parameter ``p`` in its optimizer's
        flat buffer (None when no optimizer owns it)."""
        for d in (self.dp, self.dp_partner):
            if d is not None and p in d.param_to_bucket:
                b, off = d.param_to_bucket[p]
                return b.grad[off: off + p.numel()]
        return None

    def _pp_dict(self, mb, temperature: float = 1.0, bin_=None) -> dict:
        """A micro-batch as the pipeline schedule takes it."""
        return {"ids": mb.input_ids, "pos": mb.positions, "cu": mb.cu_seqlens, "max": mb.max_seqlen,
                "labels": mb.labels, "temperature": temperature, "mb": mb, "bin": bin_}

    def _placeholder(self):
        t = Trajectory(uid=-1, request_id=-1, prompt_ids=[0], response_ids=[0], rollout_logprobs=[0.0],
                       response_mask=[0])
        return build_micro_batch([t], [0], self.device)

    # ------------------------------------------------------------- logprob
    @torch.no_grad()
    def compute_log_prob(self, trajs: list[Trajectory], idx: list[int], field: str = "old_logprobs",
                         temperature: float = 1.0) -> None:
        self.model.eval()
        if self.pp is not None:
            bins = pack_micro_batches(idx, trajs, self.max_tokens)
            mbs = [build_micro_batch(trajs, b, self.device) for b in bins]
            for mb, lp in zip(mbs, self.pp.forward_only([self._pp_dict(mb, temperature) for mb in mbs])):
                lp = lp.cpu()
                for i, sl in response_slices(mb, trajs):
                    setattr(trajs[i], field, lp[sl].tolist())
            return
        for bin_ in self._lockstep(pack_micro_batches(idx, trajs, self.max_tokens)):
            if bin_ is None:
                mb = self._placeholder()
                self.model.logprobs(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen, mb.labels, temperature)
                continue
            mb = build_micro_batch(trajs, bin_, self.device)
            if self.cp_group is not None:
                sh = self._new_shard(mb.cu_seqlens)
                lp, _ = self.model.logprobs(sh.local(mb.input_ids), sh.positions(), sh.plan, sh.plan.max_q,
                                            sh.local(mb.labels), temperature)
                lp = sh.full(lp.float())
            else:
                lp, _ = self.model.logprobs(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen, mb.labels,
                                            temperature)
            lp = lp.float().cpu()
            for i, sl in response_slices(mb, trajs):
                setattr(trajs[i], field, lp[sl].tolist())

    @torch.no_grad()
    def compute_values(self, trajs: list[Trajectory], idx: list[int]) -> None:
        if self.pp is not None:
            bins = pack_micro_batches(idx, trajs, self.max_tokens)
            mbs = [build_micro_batch(trajs, b, self.device) for b in bins]
            for mb, v in zip(mbs, self.pp.forward_only([self._pp_dict(mb) for mb in mbs])):
                v = v.cpu()
                for i, sl in response_slices(mb, trajs):
                    trajs[i].old_values = v[sl].tolist()
            return
        for bin_ in self._lockstep(pack_micro_batches(idx, trajs, self.max_tokens)):
            if bin_ is None:
                mb = self._placeholder()
                self.model.values(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen)
                continue
            mb = build_micro_batch(trajs, bin_, self.device)
            if self.cp_group is not None:
                sh = self._new_shard(mb.cu_seqlens)
                v = sh.full(self.model.values(sh.local(mb.input_ids), sh.positions(), sh.plan,
                                              sh.plan.max_q).float()).cpu()
            else:
                v = self.model.values(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen).float().cpu()
            for i, sl in response_slices(mb, trajs):
                trajs[i].old_values = v[sl].tolist()

    # -------------------------------------------------------------- update
    def _mini_batches(self, trajs: list[Trajectory]) -> list[list[int]]:
        return mini_batch_groups(trajs, int(self.cfg.actor.ppo_mini_batch_size))

    def _policy_loss(self, lp, ent, mb, shard, trajs, bin_, num_seqs, global_tokens, stats):
        """DAPO / PPO loss of one micro-batch (clip-higher, dual clip, optional
        entropy bonus, KL loss and truncated importance weights); appends the
        micro-batch's metrics to ``stats``."""
        ac = self.cfg.actor
        tis = mb.extra.get("is_weights")
        if bool(self.cfg.algorithm.rollout_correction.tis):
            rl = shard(build_micro_batch(trajs, bin_, self.device, field_old="rollout_logprobs").old_logprobs)
            w = algos.truncated_is_weight(mb.old_logprobs, rl, float(self.cfg.algorithm.rollout_correction.tis_cap))
            tis = w if tis is None else tis * w
        agg = dict(seq_ids=mb.seq_ids, num_seqs=num_seqs, global_tokens=global_tokens)
        loss, m = algos.ppo_policy_loss(lp, mb.old_logprobs, mb.advantages, mb.loss_mask,
                                        float(ac.clip_ratio_low), float(ac.clip_ratio_high),
                                        float(ac.clip_ratio_c), ac.loss_agg_mode, tis_weight=tis, **agg)
        pg_loss = loss.detach()
        if float(ac.entropy_coeff) != 0.0:
            loss = loss - float(ac.entropy_coeff) * algos.agg_loss(ent, mb.loss_mask, ac.loss_agg_mode, **agg)
        if ac.use_kl_loss:
            ref = shard(build_micro_batch(trajs, bin_, self.device, field_old="ref_logprobs").old_logprobs)
            kl = algos.kl_penalty(lp, ref, ac.kl_loss_type)
            loss = loss + float(ac.kl_loss_coef) * algos.agg_loss(kl, mb.loss_mask, ac.loss_agg_mode, **agg)
        with torch.no_grad():
            m["pg_loss"] = pg_loss
            m["entropy"] = (ent.detach() * mb.loss_mask).sum() / global_tokens
        for k, v in m.items():
            stats.setdefault(k, []).append(v)
        return loss

    def update_policy(self, trajs: list[Trajectory], temperature: float = 1.0, step_guard=None,
                      sync_every_micro_batch: bool = False, plan: list[tuple] | None = None) -> dict:
        """PPO-family update.  ``step_guard`` (a context manager) wraps each
        optimizer step, i.e. the in-place parameter update (the PS exclusive-push
        lock when a colocated rollout reads the parameters concurrently).
        ``plan`` (from :func:`plan_update`) gives this rank's share of each
        mini-batch when ``trajs`` holds only this rank's trajectories; without it
        every rank sees the whole batch and takes its token-balanced share."""
        import contextlib
        guard = step_guard if step_guard is not None else contextlib.nullcontext
        ac = self.cfg.actor
        self.model.train()
        stats: dict[str, list] = {}
        opt_s = 0.0
        if plan is None:
            plan = [(self.my_share(trajs, mini), float(sum(loss_tokens(trajs[i]) for i in mini)), len(mini))
                    for mini in self._mini_batches(trajs)]
        elif self.cfg.algorithm.rollout_correction.get("rollout_rs", None):
            plan = self._recount_plan(trajs, plan)
        for _epoch in range(int(ac.ppo_epochs)):
            for mine, global_tokens, num_seqs in plan:
                if self.pp is not None:
                    bins = pack_micro_batches(mine, trajs, self.max_tokens)
                    mbs = [self._pp_dict(build_micro_batch(trajs, b, self.device), temperature, bin_=b)
                           for b in bins]
                    self.pp.train_step(mbs, lambda lp, ent, d: self._policy_loss(
                        lp, ent, d["mb"], lambda t: t, trajs, d["bin"], num_seqs, global_tokens, stats))
                    self.pp.reduce_tied_grads(self._main_grad)
                for bin_ in (self._lockstep(pack_micro_batches(mine, trajs, self.max_tokens))
                             if self.pp is None else []):
                    if bin_ is None:
                        mb = self._placeholder()
                        lp, ent = self.model.logprobs(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen,
                                                      mb.labels, temperature)
                        ((lp * 0).sum() + (ent * 0).sum()).backward()
                        continue
                    mb = build_micro_batch(trajs, bin_, self.device)
                    shard = self._cp_shard(mb)
                    lp, ent = self.model.logprobs(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen,
                                                  mb.labels, temperature)
                    self._policy_loss(lp, ent, mb, shard, trajs, bin_, num_seqs, global_tokens, stats).backward()
                    if sync_every_micro_batch and self.device.type == "cuda":
                        # bounded launch queue: the host thread releases the GIL here
                        torch.cuda.current_stream().synchronize()
                t_opt = time.perf_counter()
                with guard():
                    st = self.dp.step(partners=[self.dp_partner] if self.dp_partner else None)
                    if self.device.type == "cuda":
                        torch.cuda.current_stream().synchronize()
                opt_s += time.perf_counter() - t_opt
                stats.setdefault("grad_norm", []).append(st["grad_norm"])
                stats.setdefault("lr", []).append(torch.tensor(st["lr"]))
        out = {}
        for k, vs in stats.items():
            t = torch.stack([v.reshape(()).float().to(self.device) for v in vs])
            out[f"actor/{k}"] = float(t.sum()) if k in ("pg_loss", "entropy") else float(t.mean())
        if self.pp is not None:
            out = self.pp.broadcast_metrics(out)
        out["timing_s/optimizer"] = opt_s
        return out

    def update_critic(self, trajs: list[Trajectory], plan: list[tuple] | None = None) -> dict:
        """Value-loss update; ``plan`` as in :meth:`update_policy`."""
        cc = self.cfg.critic
        self.model.train()
        stats: dict[str, list] = {}
        if plan is None:
            plan = [(self.my_share(trajs, mini), float(sum(loss_tokens(trajs[i]) for i in mini)), len(mini))
                    for mini in self._mini_batches(trajs)]
        def targets(mb):
            old_v = torch.zeros(mb.num_tokens, dtype=torch.float32, device=self.device)
            ret = torch.zeros_like(old_v)
            for j, (i, sl) in enumerate(response_slices(mb, trajs)):
                old_v[sl] = torch.tensor(trajs[i].old_values, device=old_v.device)
                ret[sl] = torch.tensor(trajs[i].returns, device=old_v.device)
            return old_v, ret

        def vloss(v, old_v, ret, mb, global_tokens):
            old_v, ret = old_v.to(v.dtype), ret.to(v.dtype)
            loss, m = algos.value_loss(v, old_v, ret, mb.loss_mask, float(cc.cliprange_value),
                                       global_tokens=global_tokens)
            m["vf_loss"] = loss.detach()
            for k, val in m.items():
                stats.setdefault(k, []).append(val)
            return loss

        for mine, global_tokens, _ in plan:
            if self.pp is not None:
                mbs = [self._pp_dict(build_micro_batch(trajs, b, self.device), bin_=b)
                       for b in pack_micro_batches(mine, trajs, self.max_tokens)]
                self.pp.train_step(mbs, lambda v, _e, d, gt=global_tokens: vloss(v, *targets(d["mb"]), d["mb"], gt))
            for bin_ in (self._lockstep(pack_micro_batches(mine, trajs, self.max_tokens))
                         if self.pp is None else []):
                if bin_ is None:
                    mb = self._placeholder()
                    (self.model.values(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen) * 0).sum().backward()
                    continue
                mb = build_micro_batch(trajs, bin_, self.device)
                old_v, ret = targets(mb)
                shard = self._cp_shard(mb)
                old_v, ret = shard(old_v), shard(ret)
                v = self.model.values(mb.input_ids, mb.positions, mb.cu_seqlens, mb.max_seqlen)
                vloss(v, old_v, ret, mb, global_tokens).backward()
            st = self.dp.step(partners=[self.dp_partner] if self.dp_partner else None)
            stats.setdefault("grad_norm", []).append(st["grad_norm"])
        out = {f"critic/{k}": float(torch.stack([x.reshape(()).float() for x in vs]).mean()) for k, vs in stats.items()}
        return self.pp.broadcast_metrics(out) if self.pp is not None else out

    # --------------------------------------------------------------- state
    def named_parameters(self) -> dict[str, torch.Tensor]:
        return {n: p.detach() for n, p in self.model.named_parameters()}
