"""Rollout engine: paged-KV continuous batching on one GPU (the vLLM role, N2).

Per :meth:`RolloutEngine.step` the scheduler either runs one *prefill* step
(chunked, up to ``max_num_batched_tokens`` new tokens over several waiting
requests, reusing cached prefix blocks) or one *decode* step over every running
sequence.  Decode runs as a replay of a CUDA graph captured per batch-size
bucket: embedding, 36x(RMSNorm, QKV GEMM, RoPE + KV-cache write, split-KV
paged decode attention, O GEMM, RMSNorm, gate_up GEMM, SwiGLU, down GEMM),
final norm, LM head and the fused sampler — one launch from the host.

Semantics needed by asynchronous RL:

* forced-length generation (``ignore_eos`` + per-request ``max_tokens``);
* per-token log-probabilities of the sampled tokens (the rollout log-probs used
  as old log-probs / for TIS);
* per-token weight version; :meth:`load_weights` bumps the version and, unless
  ``keep_kv``, re-queues in-flight requests for re-prefill with the new weights
  (partial rollout across versions);
* :meth:`abort` returns the partial trajectory so the caller can resume it
  elsewhere (migration).
"""

from __future__ import annotations

import math
import time
from collections import deque
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..ops.linear import decode_gate_up_swiglu, decode_linear, gate_up_swiglu
from ..ops.linear import linear as linear_tc
from ..utils import transfer
from ..models.config import ModelArgs
from .kv_cache import BlockManager, allocate_kv_tensors


@dataclass
class SamplingParams:
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_tokens: int = 128
    ignore_eos: bool = False
    stop_token_ids: tuple = ()
    seed: int = 0


@dataclass
class GenRequest:
    request_id: int
    prompt_ids: list
    params: SamplingParams
    version_tag: int = 0
    meta: dict = field(default_factory=dict)
    # resumed partial output (partial rollout / migration)
    prev_output_ids: list = field(default_factory=list)
    prev_logprobs: list = field(default_factory=list)
    prev_versions: list = field(default_factory=list)


@dataclass
class RequestOutput:
    request_id: int
    prompt_ids: list
    output_ids: list
    logprobs: list
    versions: list
    finish_reason: str          # length | stop | abort
    version_tag: int
    meta: dict
    num_cached_tokens: int = 0


class _Seq:
    __slots__ = ("req", "tokens", "n_prompt", "out_ids", "out_lp", "out_ver", "blocks", "num_computed", "row",
                 "cached_tokens", "arrival", "registered_blocks")

    def __init__(self, req: GenRequest):
        self.req = req
        self.n_prompt = len(req.prompt_ids)
        self.tokens = list(req.prompt_ids) + list(req.prev_output_ids)
        self.out_ids = list(req.prev_output_ids)
        self.out_lp = list(req.prev_logprobs)
        self.out_ver = list(req.prev_versions)
        self.blocks: list[int] = []
        self.num_computed = 0
        self.row = -1
        self.cached_tokens = 0
        self.arrival = time.monotonic()
        self.registered_blocks = 0

    def remaining(self) -> int:
        return self.req.params.max_tokens - len(self.out_ids)


class EngineWeights:
    """Inference weights in the fused layout (TP=1 shapes equal the trainer's)."""

    def __init__(self, args: ModelArgs, device, dtype=torch.bfloat16):
        self.args = args
        self.device = torch.device(device)
        self.dtype = dtype
        self.tensors: dict[str, torch.Tensor] = {}

    @classmethod
    def from_model(cls, model, device=None, dtype=torch.bfloat16, share: bool = False) -> "EngineWeights":
        dev = device or next(model.parameters()).device
        w = cls(model.args, dev, dtype)
        for name, p in model.named_parameters():
            t = p.detach()
            w.tensors[name] = t if share and t.device == w.device and t.dtype == dtype else \
                t.to(device=dev, dtype=dtype).contiguous().clone()
        for name, b in model.named_buffers():
            w.tensors[name] = b.to(dev)
        return w

    def __getitem__(self, k):
        return self.tensors[k]

    def get(self, k):
        return self.tensors.get(k)

    @torch.no_grad()
    def copy_from_state(self, state: dict[str, torch.Tensor]) -> None:
        for k, t in state.items():
            if k in self.tensors:
                self.tensors[k].copy_(t, non_blocking=True)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors.values())

    def lm_head(self) -> torch.Tensor:
        return self.tensors["embed.weight"] if self.args.tie_word_embeddings else self.tensors["lm_head.weight"]

    @torch.no_grad()
    def move_to_pool(self, pool, tag: str = "weights") -> None:
        """Re-home every tensor in a virtual-memory region of ``pool`` (same
        values, new addresses) so the engine's weights can be released and
        restored around a sleep."""
        items = [(k, t) for k, t in self.tensors.items() if t.is_cuda]
        offs, total = [], 0
        for _, t in items:
            total = (total + 255) // 256 * 256            # 256-byte aligned views
            offs.append(total)
            total += t.numel() * t.element_size()
        flat = pool.tensor(tag, (total,), torch.uint8)    # one region for every tensor
        for (k, t), off in zip(items, offs):
            nb = t.numel() * t.element_size()
            dst = flat[off:off + nb].view(t.dtype).view(t.shape)
            dst.copy_(t)
            self.tensors[k] = dst


def _nullctx():
    import contextlib
    return contextlib.nullcontext()


class RolloutEngine:
    def __init__(self, args: ModelArgs, weights: EngineWeights, *, max_num_seqs: int = 256,
                 max_model_len: int = 8192 + 1024, block_size: int = 64, max_num_batched_tokens: int = 10240,
                 kv_cache_gb: float | None = None, num_blocks: int | None = None, enable_prefix_caching: bool = True,
                 use_cuda_graph: bool = True, keep_kv_on_update: bool = False, version: int = 0,
                 eos_token_id: int | None = None, tp=None, memory_pool=None, decode_gemm: str = "library",
                 kv_offload_blocks: int = 0):
        # tensor parallelism (``tp``: parallel.tp.TPGroup): this engine holds query heads,
        # KV heads and MLP columns [r/P, (r+1)/P) of every layer (weights in the same
        # layout as the TP trainer's shards) and its KV cache for its own KV heads; the
        # O and down projections end in an all-reduce over the TP group.  Every TP rank
        # runs the same schedule (the caller feeds them identical requests), so the
        # replicated LM head gives identical logits and identical sampled tokens.
        self.tp = tp
        self.full_args = args
        if tp is not None and tp.world > 1:
            if args.qk_norm_full or args.hidden_act != "silu":
                raise NotImplementedError("tensor-parallel rollout of full-width q/k norms or GeGLU is not implemented")
            if args.is_moe and (args.num_experts % tp.world or args.shared_expert_intermediate_size % tp.world):
                raise ValueError("expert parallelism over the TP group needs experts (and the shared expert's "
                                 "width) divisible by the TP size")
            from dataclasses import replace
            if args.num_heads % tp.world or (args.num_kv_heads % tp.world and tp.world % args.num_kv_heads):
                raise ValueError(f"{args.num_heads} query / {args.num_kv_heads} KV heads do not split over "
                                 f"TP={tp.world}")
            # more TP ranks than KV heads: each rank keeps the one KV head its query
            # heads read (replicated over the tp.world / nkv ranks that share it)
            # MoE: expert parallelism follows TP: rank r holds experts [r E/P, (r+1) E/P)
            # at full width (routing still spans all E experts) and 1/P of the
            # shared expert's width; its partial output joins the MLP all-reduce
            args = replace(args, num_heads=args.num_heads // tp.world,
                           num_kv_heads=max(1, args.num_kv_heads // tp.world),
                           intermediate_size=args.intermediate_size // tp.world,
                           shared_expert_intermediate_size=args.shared_expert_intermediate_size // tp.world)
        else:
            self.tp = None
        self.args = args
        self.w = weights
        self.device = weights.device
        self.dtype = weights.dtype
        self.max_num_seqs = int(max_num_seqs)
        self.max_model_len = int(max_model_len)
        args.check_context(self.max_model_len)
        self.block_size = int(block_size)
        self.max_blocks_per_seq = math.ceil(self.max_model_len / self.block_size)
        self.max_num_batched_tokens = int(max_num_batched_tokens)
        self.enable_prefix_caching = enable_prefix_caching
        self.keep_kv_on_update = keep_kv_on_update
        self.version = int(version)
        self.eos_token_id = eos_token_id
        a = args
        per_block = 2 * a.num_layers * a.num_kv_heads * self.block_size * a.head_dim * torch.finfo(self.dtype).bits // 8
        if num_blocks is None:
            gb = kv_cache_gb if kv_cache_gb is not None else 4.0
            num_blocks = max(2 * self.max_blocks_per_seq, int(gb * (1 << 30) // per_block))
        self.num_blocks = int(num_blocks)
        self.bm = BlockManager(self.num_blocks, self.block_size)
        self.bm.set_version(self.version)
        # memory_pool (parallel.memory.MemoryPool): KV cache and weights in
        # virtual-memory regions ("kv", "weights") so sleep() can release them
        self.pool = memory_pool
        self.asleep = False
        # decode-step projections: "library" (cuBLAS through torch; faster on
        # B200 at every batch size measured so far) or "tcgen05" (the
        # weight-streaming / split-K kernels of csrc/gemm_skinny.cu, gemm_2sm.cu)
        if decode_gemm not in ("library", "tcgen05"):
            raise ValueError(f"decode_gemm must be 'library' or 'tcgen05', not {decode_gemm!r}")
        self.decode_gemm = decode_gemm
        # host KV store (C29): a preempted sequence's complete blocks are copied to
        # pinned host memory (keyed by their chained content hashes) and copied
        # back when it resumes, instead of being recomputed
        self.offload = None
        if memory_pool is not None:
            weights.move_to_pool(memory_pool, "weights")
        self.k_cache, self.v_cache = allocate_kv_tensors(a.num_layers, self.num_blocks, a.num_kv_heads,
                                                         self.block_size, a.head_dim, self.dtype, self.device,
                                                         pool=memory_pool)
        if int(kv_offload_blocks) > 0:
            from .kv_offload import KVOffloadStore
            self.offload = KVOffloadStore(self, int(kv_offload_blocks))
        self.waiting: deque[_Seq] = deque()
        self.running: list[_Seq] = []
        self.by_id: dict[int, _Seq] = {}
        self.finished_unreported: list[RequestOutput] = []
        self.is_cuda = self.device.type == "cuda"
        self.use_cuda_graph = use_cuda_graph and self.is_cuda
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._graph_launches: dict[int, int] = {}
        self._graph_pool = None
        self._alloc_static()
        # stats
        self.stats = {"prefill_tokens": 0, "decode_tokens": 0, "prefill_steps": 0, "decode_steps": 0,
                      "preemptions": 0, "cached_tokens": 0, "prefill_time": 0.0, "decode_time": 0.0,
                      "offloaded_blocks": 0, "onloaded_blocks": 0, "migrated_out": 0, "migrated_in": 0}

    # ------------------------------------------------------------- buffers
    def _alloc_static(self):
        B, MB = self.max_num_seqs, self.max_blocks_per_seq
        dev = self.device
        self.s_tokens = torch.zeros(B, dtype=torch.long, device=dev)
        self.s_pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_slots = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_bt = torch.zeros(B, MB, dtype=torch.int32, device=dev)
        self.s_temps = torch.ones(B, dtype=torch.float32, device=dev)
        self.s_seeds = torch.zeros(B, dtype=torch.long, device=dev)
        self.s_out_tok = torch.zeros(B, dtype=torch.long, device=dev)
        self.s_out_lp = torch.zeros(B, dtype=torch.float32, device=dev)
        pin = self.is_cuda
        self.h_tokens = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        self.h_pos = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_slots = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_lens = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.h_bt = torch.zeros(B, MB, dtype=torch.int32, pin_memory=pin)
        self.h_temps = torch.ones(B, dtype=torch.float32, pin_memory=pin)
        self.h_seeds = torch.zeros(B, dtype=torch.long, pin_memory=pin)
        # two output buffers: the host reads one step's samples while the next is copied
        self._h_out = [(torch.zeros(B, dtype=torch.long, pin_memory=pin),
                        torch.zeros(B, dtype=torch.float32, pin_memory=pin)) for _ in range(2)]
        self._out_flip = 0
        self._pending = None
        self._h2d_done = None
        self.n_bt = self.h_bt.numpy()
        a = self.args
        self.max_splits = 1
        if self.is_cuda:
            self.max_splits = 32
            self.decode_scratch = torch.empty(B * a.num_heads * self.max_splits * (a.head_dim + 1),
                                              dtype=torch.float32, device=dev)

    # ----------------------------------------------------------- requests
    def add_request(self, req: GenRequest) -> None:
        if self.asleep:
            raise RuntimeError("engine is asleep: wake() it before adding requests")
        if req.request_id in self.by_id:
            raise ValueError(f"duplicate request id {req.request_id}")
        total = len(req.prompt_ids) + len(req.prev_output_ids)
        if total >= self.max_model_len:
            raise ValueError(f"request {req.request_id}: {total} tokens >= max_model_len {self.max_model_len}")
        s = _Seq(req)
        self.by_id[req.request_id] = s
        self.waiting.append(s)

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)

    def num_unfinished(self) -> int:
        return len(self.waiting) + len(self.running)

    def _output(self, s: _Seq, reason: str) -> RequestOutput:
        return RequestOutput(s.req.request_id, list(s.req.prompt_ids), list(s.out_ids), list(s.out_lp),
                             list(s.out_ver), reason, s.req.version_tag, s.req.meta, s.cached_tokens)

    def _free(self, s: _Seq, register: bool) -> None:
        if register and self.enable_prefix_caching and s.blocks:
            self.bm.register_full_blocks(s.blocks, s.tokens[: s.num_computed], s.registered_blocks)
        self.bm.release(s.blocks)
        s.blocks = []

    def _remove_running(self, s: _Seq) -> None:
        i = s.row
        last = self.running[-1]
        self.running[i] = last
        last.row = i
        self.running.pop()
        if last is not s:
            self._write_bt_row(last)
        s.row = -1

    def abort(self, request_id: int) -> RequestOutput | None:
        """Stop a request and return its partial output (or None if unknown)."""
        self._drain(self.finished_unreported)
        s = self.by_id.pop(request_id, None)
        if s is None:
            return None
        if s.row >= 0:
            self._remove_running(s)
        else:
            try:
                self.waiting.remove(s)
            except ValueError:
                pass
        self._free(s, register=False)
        return self._output(s, "abort")

    def migrate_request(self, request_id: int, dst: "RolloutEngine") -> bool:
        """Move a request to engine ``dst`` together with the KV of every token
        computed so far (the KV block kernel copies the blocks: same GPU, a
        peer GPU over NVLink, or host memory), so ``dst`` continues it with a
        one-token prefill instead of recomputing the context.  Both engines must
        hold the same weight version.  Returns False (and keeps the request) when
        ``dst`` has no room."""
        from .kv_offload import transfer_direct
        self._drain(self.finished_unreported)
        dst._drain(dst.finished_unreported)
        s = self.by_id.get(request_id)
        bs = self.block_size
        if s is None or dst is self or dst.asleep or dst.version != self.version or dst.block_size != bs:
            return False
        need = -(-s.num_computed // bs)
        if dst.num_unfinished() >= dst.max_num_seqs or not dst.bm.can_allocate(need + 1):
            return False
        new = dst.bm.allocate(need)
        if need:
            cross = self.is_cuda and dst.is_cuda and self.device != dst.device
            if self.is_cuda:
                ready = torch.cuda.Event()
                ready.record(torch.cuda.current_stream(self.device))     # the source's KV writes
                torch.cuda.current_stream(dst.device).wait_event(ready)
            if cross:
                with torch.cuda.device(dst.device):
                    ops.ext().enable_peer_access(self.device.index)
            with torch.cuda.device(dst.device) if dst.is_cuda else _nullctx():
                transfer_direct(self, dst, s.blocks[:need], new)
            if self.is_cuda:
                done = torch.cuda.Event()
                done.record(torch.cuda.current_stream(dst.device))       # before the source reuses its blocks
                torch.cuda.current_stream(self.device).wait_event(done)
        self.by_id.pop(request_id)
        if s.row >= 0:
            self._remove_running(s)
        else:
            self.waiting.remove(s)
        self._free(s, register=False)
        s.blocks = new
        s.registered_blocks = 0
        dst.by_id[request_id] = s
        dst.waiting.appendleft(s)
        self.stats["migrated_out"] += 1
        dst.stats["migrated_in"] += 1
        return True

    def abort_all(self) -> list[RequestOutput]:
        return [o for o in (self.abort(r) for r in list(self.by_id)) if o is not None]

    # ------------------------------------------------------- sleep / wake
    def sleep(self, keep_weights: bool = True) -> tuple[list[RequestOutput], int]:
        """Release this engine's GPU memory for another role (elastic time
        sharing; the reference's vLLM sleep levels 1 and 2).  In-flight requests
        are interrupted and returned (their partial outputs can resume elsewhere
        or after wake).  The KV cache's physical memory is released and its
        contents dropped (the prefix cache is cleared); the weights' memory is
        released too, with a pinned host copy if ``keep_weights`` (level 1),
        else dropped (level 2: load weights after :meth:`wake`).  Addresses are
        kept, so captured decode graphs stay valid.  Returns (interrupted
        outputs, bytes released)."""
        if self.pool is None:
            raise RuntimeError("sleep needs an engine built with a memory_pool")
        if self.asleep:
            return [], 0
        outs = self.abort_all()
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        freed = self.pool.sleep("kv", backup=False) + self.pool.sleep("weights", backup=keep_weights)
        self.bm = BlockManager(self.num_blocks, self.block_size)
        self.bm.set_version(self.version)
        if self.offload is not None:
            self.offload.clear()
        self.asleep = True
        return outs, freed

    def wake(self) -> int:
        """Map memory back at the same addresses (weights restored from the
        host copy when one was kept; the KV cache starts empty)."""
        if not self.asleep:
            return 0
        n = self.pool.wake("weights") + self.pool.wake("kv")
        self.asleep = False
        return n

    # ------------------------------------------------------------- weights
    @torch.no_grad()
    def load_weights(self, state: dict | None, version: int) -> None:
        """Install new weights (``state`` may be None when the caller already
        wrote them in place) and advance the weight version."""
        self._drain(self.finished_unreported)
        if state:
            self.w.copy_from_state(state)
        self.version = int(version)
        if not self.keep_kv_on_update:
            # re-prefill every in-flight sequence with the new weights
            for s in list(self.running):
                self._remove_running(s)
                self._free(s, register=False)
                s.num_computed = 0
                s.req.version_tag = max(s.req.version_tag, self.version)
                self.waiting.appendleft(s)
            for s in self.waiting:
                if s.blocks:
                    self._free(s, register=False)
                    s.num_computed = 0
            self.bm.set_version(self.version)
            if self.offload is not None:
                self.offload.clear()            # host copies hold the old weights' KV

    # --------------------------------------------------------------- step
    def step(self) -> list[RequestOutput]:
        """Run one scheduling step; returns requests that finished in it (and
        any that finished while an abort or a weight load completed the step in
        flight)."""
        out: list[RequestOutput] = self.finished_unreported
        self.finished_unreported = []
        if self.waiting and len(self.running) < self.max_num_seqs:
            self._drain(out)                  # admission changes the batch: finish the step in flight
            did = self._prefill_step(out)
            if did:
                return out
        if self.running:
            self._decode_step(out)
        else:
            self._drain(out)
        return out

    def _finish_check(self, s: _Seq, tok: int) -> str | None:
        p = s.req.params
        if len(s.out_ids) >= p.max_tokens:
            return "length"
        if not p.ignore_eos and ((self.eos_token_id is not None and tok == self.eos_token_id)
                                 or tok in p.stop_token_ids):
            return "stop"
        if len(s.tokens) >= self.max_model_len:
            return "length"
        return None

    def _append(self, s: _Seq, tok: int, lp: float, out: list) -> bool:
        s.tokens.append(tok)
        s.out_ids.append(tok)
        s.out_lp.append(lp)
        s.out_ver.append(self.version)
        reason = self._finish_check(s, tok)
        if reason:
            if s.row >= 0:
                self._remove_running(s)
            self.by_id.pop(s.req.request_id, None)
            self._free(s, register=True)
            out.append(self._output(s, reason))
            return True
        return False

    # ------------------------------------------------------------- prefill
    def _prefill_step(self, out: list) -> bool:
        bs = self.block_size
        budget = self.max_num_batched_tokens
        batch: list[tuple[_Seq, int]] = []
        while self.waiting and budget > 0 and len(self.running) + len(batch) < self.max_num_seqs:
            s = self.waiting[0]
            if not s.blocks and self.enable_prefix_caching and s.num_computed == 0:
                blocks = self.bm.match_prefix(s.tokens)
                # always recompute at least the last token
                while blocks and len(blocks) * bs >= len(s.tokens):
                    self.bm.release([blocks.pop()])
                s.blocks = blocks
                s.num_computed = len(blocks) * bs
                s.cached_tokens = s.num_computed
                s.registered_blocks = len(blocks)
                self.stats["cached_tokens"] += s.num_computed
            if self.offload is not None and s.num_computed == len(s.blocks) * bs:
                self._onload(s)
            todo = len(s.tokens) - s.num_computed
            chunk = min(todo, budget)
            need = math.ceil((s.num_computed + chunk) / bs) - len(s.blocks)
            # reserve room for the request to keep decoding a while
            if not self.bm.can_allocate(need + (1 if chunk == todo else 0)):
                if not batch and not self.running:
                    raise MemoryError("KV cache too small for a single request")
                break
            s.blocks.extend(self.bm.allocate(need))
            self.waiting.popleft()
            batch.append((s, chunk))
            budget -= chunk
        if not batch:
            return False
        t0 = time.perf_counter()
        self._run_prefill(batch, out)
        self.stats["prefill_time"] += time.perf_counter() - t0
        self.stats["prefill_steps"] += 1
        return True

    @torch.no_grad()
    def _run_prefill(self, batch, out):
        a, bs, dev = self.args, self.block_size, self.device
        ids, pos, slots, cu, lens = [], [], [], [0], []
        bt = np.zeros((len(batch), self.max_blocks_per_seq), dtype=np.int32)
        for i, (s, n) in enumerate(batch):
            p0 = s.num_computed
            ids.extend(s.tokens[p0: p0 + n])
            pr = np.arange(p0, p0 + n)
            pos.append(pr)
            blk = np.asarray(s.blocks, dtype=np.int64)
            slots.append(blk[pr // bs] * bs + pr % bs)
            cu.append(cu[-1] + n)
            lens.append(p0 + n)
            bt[i, : len(s.blocks)] = s.blocks
        T = cu[-1]
        t_ids = torch.tensor(ids, dtype=torch.long).to(dev, non_blocking=True)
        t_pos = torch.from_numpy(np.concatenate(pos).astype(np.int32)).to(dev, non_blocking=True)
        t_slots = torch.from_numpy(np.concatenate(slots).astype(np.int32)).to(dev, non_blocking=True)
        t_cu = torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True)
        t_lens = torch.tensor(lens, dtype=torch.int32).to(dev, non_blocking=True)
        t_bt = torch.from_numpy(bt).to(dev, non_blocking=True)
        max_q = max(n for _, n in batch)
        transfer.h2d(T * 16 + 8 * len(cu) + bt.nbytes)
        h = self._forward(t_ids, t_pos, t_slots, mode="prefill", cu_q=t_cu, kv_lens=t_lens, block_table=t_bt,
                          max_q=max_q)
        # sample for sequences whose prompt is now fully computed
        done_rows, done_seqs = [], []
        for i, (s, n) in enumerate(batch):
            s.num_computed += n
            if s.num_computed == len(s.tokens):
                done_rows.append(cu[i + 1] - 1)
                done_seqs.append(s)
            else:
                self.waiting.appendleft(s)   # continue chunked prefill next step
        self.stats["prefill_tokens"] += T
        if done_seqs:
            rows = torch.tensor(done_rows, dtype=torch.long, device=dev)
            logits = F.linear(h.index_select(0, rows), self.w.lm_head())
            temps = torch.tensor([s.req.params.temperature for s in done_seqs], dtype=torch.float32, device=dev)
            seeds = torch.tensor([s.req.params.seed for s in done_seqs], dtype=torch.long, device=dev)
            streams = torch.tensor([len(s.tokens) for s in done_seqs], dtype=torch.int32, device=dev)
            p0 = done_seqs[0].req.params
            tok, lp = ops.sample(logits, temps, seeds, streams, top_k=p0.top_k, top_p=p0.top_p)
            tok, lp = tok.tolist(), lp.tolist()
            transfer.h2d(20 * len(done_seqs))
            transfer.d2h(12 * len(done_seqs))
            for s, t, l in zip(done_seqs, tok, lp):
                if self.enable_prefix_caching:
                    self.bm.register_full_blocks(s.blocks, s.tokens[: s.num_computed], s.registered_blocks)
                    s.registered_blocks = s.num_computed // self.block_size
                s.row = len(self.running)
                self.running.append(s)
                self._write_bt_row(s)
                self._append(s, t, l, out)

    def _write_bt_row(self, s: _Seq):
        r = s.row
        self.n_bt[r, : len(s.blocks)] = s.blocks

    # -------------------------------------------------------------- decode
    def _ensure_decode_slots(self) -> None:
        bs = self.block_size
        for s in list(self.running):
            if s.row < 0:                      # preempted earlier in this loop
                continue
            pos = len(s.tokens) - 1            # position of the token being fed
            if pos // bs >= len(s.blocks):
                while not self.bm.can_allocate(1):
                    victim = self.running[-1]
                    self._preempt(victim)
                    if victim is s:
                        break
                if s.row < 0:
                    continue
                s.blocks.extend(self.bm.allocate(1))
                self.n_bt[s.row, len(s.blocks) - 1] = s.blocks[-1]

    def _onload(self, s: _Seq) -> None:
        """Resume from the host KV store: the complete blocks after the device
        prefix whose content hashes the store holds are copied back (the last
        token is always recomputed)."""
        bs = self.block_size
        hs = self.bm.chain_hashes(s.tokens)
        i0 = len(s.blocks)
        k = 0
        while i0 + k < len(hs) and hs[i0 + k] in self.offload.index and (i0 + k + 1) * bs < len(s.tokens):
            k += 1
        if k == 0 or not self.bm.can_allocate(k + 1):
            return
        new = self.bm.allocate(k)
        n = self.offload.onload(hs[i0: i0 + k], new)
        if n < k:
            self.bm.release(new[n:])
            new = new[:n]
        s.blocks.extend(new)
        s.num_computed += n * bs
        s.cached_tokens += n * bs
        self.stats["onloaded_blocks"] += n

    def _preempt(self, s: _Seq) -> None:
        self._remove_running(s)
        if self.offload is not None and s.blocks:
            full = min(s.num_computed // self.block_size, len(s.blocks))
            if full:
                hs = self.bm.chain_hashes(s.tokens[: full * self.block_size])
                self.stats["offloaded_blocks"] += self.offload.offload(hs, s.blocks[:full])
        self._free(s, register=False)
        s.num_computed = 0
        self.waiting.appendleft(s)
        self.stats["preemptions"] += 1

    def _bucket(self, n: int) -> int:
        for b in (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512):
            if b >= n:
                return min(b, self.max_num_seqs)
        return self.max_num_seqs

    # A decode step in flight (CUDA graphs only): its rows, batch sizes, output
    # buffers and completion event.  When no running sequence can finish with the
    # token it computes and nothing waits for admission, the next step is
    # launched before this one's tokens reach the host (its input tokens are
    # copied on the device from the sampler's output), and the host appends
    # this step's tokens while the GPU runs the next: the host's per-step work
    # hides behind the device's.
    def _chainable(self) -> bool:
        if self._pending is None or self.waiting:
            return False
        new_blocks = 0
        bs = self.block_size
        for s in self.running:
            p = s.req.params
            if len(s.out_ids) + 2 > p.max_tokens or len(s.tokens) + 2 > self.max_model_len:
                return False
            if not p.ignore_eos and (self.eos_token_id is not None or p.stop_token_ids):
                return False
            if len(s.tokens) // bs >= len(s.blocks):
                new_blocks += 1
        return self.bm.can_allocate(new_blocks)

    def _drain(self, out: list) -> None:
        """Append the tokens of the step in flight (if any)."""
        if self._pending is not None:
            pend, self._pending = self._pending, None
            self._finish(pend, out)

    def _finish(self, pend, out: list) -> None:
        rows, B, nb, tok_buf, lp_buf, done = pend
        if done is not None:
            done.synchronize()
            transfer.d2h(nb * 12)
            tok = tok_buf.numpy()[:B].tolist()
            lp = lp_buf.numpy()[:B].tolist()
        else:
            tok = self.s_out_tok[:B].tolist()
            lp = self.s_out_lp[:B].tolist()
        for s, t, l in zip(rows, tok, lp):
            s.num_computed = len(s.tokens)
            self._append(s, t, l, out)
        self.stats["decode_tokens"] += B
        self.stats["decode_steps"] += 1

    def _launch(self, chained: bool):
        """Prepare and launch one decode step over the running sequences;
        ``chained``: the previous step's tokens are not appended yet (each
        sequence is one position further than its token list says)."""
        if self._h2d_done is not None:
            self._h2d_done.synchronize()      # the last step's host->device copies read these buffers
        shift = 1 if chained else 0
        if not chained:
            self._ensure_decode_slots()
        else:
            bs = self.block_size
            for s in self.running:            # room checked by _chainable: no preemption here
                if len(s.tokens) // bs >= len(s.blocks):
                    s.blocks.extend(self.bm.allocate(1))
                    self.n_bt[s.row, len(s.blocks) - 1] = s.blocks[-1]
        B = len(self.running)
        if B == 0:
            return None
        bs = self.block_size
        pos = np.fromiter((len(s.tokens) - 1 + shift for s in self.running), dtype=np.int32, count=B)
        blk = np.fromiter((s.blocks[p // bs] for s, p in zip(self.running, pos)), dtype=np.int64, count=B)
        slots = (blk * bs + pos % bs).astype(np.int32)
        nb = self._bucket(B)
        if not chained:
            self.h_tokens.numpy()[:B] = np.fromiter((s.tokens[-1] for s in self.running), dtype=np.int64, count=B)
        self.h_pos.numpy()[:B] = pos
        self.h_slots.numpy()[:B] = slots
        self.h_lens.numpy()[:B] = pos + 1
        self.h_temps.numpy()[:B] = [s.req.params.temperature for s in self.running]
        self.h_seeds.numpy()[:B] = [s.req.params.seed for s in self.running]
        if nb > B:
            # padded rows: length-1 context in block 0 of a harmless slot; results ignored
            self.h_tokens.numpy()[B:nb] = 0
            self.h_pos.numpy()[B:nb] = 0
            self.h_slots.numpy()[B:nb] = -1
            self.h_lens.numpy()[B:nb] = 1
            self.n_bt[B:nb, 0] = 0
        if chained:
            self.s_tokens[:nb].copy_(self.s_out_tok[:nb])    # the previous step's samples, on the device
        else:
            self.s_tokens[:nb].copy_(self.h_tokens[:nb], non_blocking=True)
        for src, dst in ((self.h_pos, self.s_pos), (self.h_slots, self.s_slots), (self.h_lens, self.s_lens),
                         (self.h_temps, self.s_temps), (self.h_seeds, self.s_seeds)):
            dst[:nb].copy_(src[:nb], non_blocking=True)
        mb = max(len(s.blocks) for s in self.running)
        self.s_bt[:nb, :mb].copy_(self.h_bt[:nb, :mb], non_blocking=True)
        transfer.h2d(nb * (4 + 4 + 4 + 4 + 8 + 4 * mb) + (0 if chained else 8 * nb))
        if self.is_cuda:
            self._h2d_done = torch.cuda.Event()
            self._h2d_done.record()
            torch.cuda.nvtx.range_push("decode_step")
        if self.use_cuda_graph:
            g = self._graphs.get(nb)
            if g is None:
                g = self._capture(nb)
            g.replay()
            ops._ext.add_launches(self._graph_launches[nb])
        else:
            self._decode_forward(nb)
        rows = list(self.running)
        if not self.is_cuda:
            return rows, B, nb, None, None, None
        torch.cuda.nvtx.range_pop()
        self._out_flip ^= 1
        tok_buf, lp_buf = self._h_out[self._out_flip]
        tok_buf[:nb].copy_(self.s_out_tok[:nb], non_blocking=True)
        lp_buf[:nb].copy_(self.s_out_lp[:nb], non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        return rows, B, nb, tok_buf, lp_buf, done

    @torch.no_grad()
    def _decode_step(self, out: list) -> None:
        t0 = time.perf_counter()
        if self.use_cuda_graph and self._chainable():
            prev = self._pending
            self._pending = self._launch(chained=True)     # the GPU runs it while the host appends prev
            self._finish(prev, out)
        else:
            self._drain(out)
            if self.running:
                pend = self._launch(chained=False)
                if pend is not None:
                    if self.use_cuda_graph:
                        self._pending = pend
                    else:
                        self._finish(pend, out)
        self.stats["decode_time"] += time.perf_counter() - t0

    def _decode_forward(self, nb: int) -> None:
        splits = 1
        if self.is_cuda:
            splits = ops.attention.decode_splits(nb, self.args.num_kv_heads, self.max_model_len)
            splits = min(splits, self.max_splits)
        h = self._forward(self.s_tokens[:nb], self.s_pos[:nb], self.s_slots[:nb], mode="decode",
                          kv_lens=self.s_lens[:nb], block_table=self.s_bt[:nb], splits=splits)
        use_tc = self.is_cuda and self.tp is None and self.decode_gemm == "tcgen05"
        w_head = self.w.lm_head()
        logits = decode_linear(h, w_head) if use_tc else F.linear(h, w_head)
        tok, lp = ops.sample(logits, self.s_temps[:nb], self.s_seeds[:nb], self.s_pos[:nb] + 1)
        self.s_out_tok[:nb].copy_(tok)
        self.s_out_lp[:nb].copy_(lp)

    def _capture(self, nb: int):
        # warm up on a side stream, then capture
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._decode_forward(nb)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        before = ops._ext.launches()
        # thread-local capture: a trainer thread may be launching work concurrently
        with torch.cuda.graph(g, pool=self._graph_pool, capture_error_mode="thread_local"):
            self._decode_forward(nb)
        self._graph_launches[nb] = ops._ext.launches() - before
        self._graphs[nb] = g
        return g

    def capture_all(self) -> None:
        """Capture the decode graph of every batch bucket up front (before any
        concurrent work starts on the device)."""
        if not self.use_cuda_graph:
            return
        for b in (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512):
            nb = min(b, self.max_num_seqs)
            if nb not in self._graphs:
                self.h_lens.numpy()[:nb] = 1
                self.h_slots.numpy()[:nb] = -1
                self.s_lens[:nb].copy_(self.h_lens[:nb])
                self.s_slots[:nb].copy_(self.h_slots[:nb])
                self.s_bt[:nb].zero_()
                self._capture(nb)
            if b >= self.max_num_seqs:
                break

    # ------------------------------------------------------------- forward
    def _forward(self, ids, pos, slots, *, mode, cu_q=None, kv_lens=None, block_table=None, max_q=0, splits=1):
        a, W = self.args, self.w
        # prefill chunks (hundreds to thousands of rows) run on the paired
        # tcgen05 GEMM with SwiGLU fused into the gate_up epilogue; decode
        # steps (one row per sequence) keep the batched library GEMM
        big = mode == "prefill" and self.is_cuda and ids.shape[0] >= 256 and self.tp is None
        if big:
            def proj(x, w, b=None):
                return linear_tc(x, w, b)

            def mlp_act(x, w):
                return gate_up_swiglu(x, w)
        elif mode == "decode" and self.is_cuda and self.tp is None and self.decode_gemm == "tcgen05":
            # one row per sequence: the weight-streaming tcgen05 kernel (split K
            # reduced in-cluster), SwiGLU fused into the gate_up epilogue
            def proj(x, w, b=None):
                return decode_linear(x, w, b)

            def mlp_act(x, w):
                return decode_gate_up_swiglu(x, w)
        else:
            def proj(x, w, b=None):
                return F.linear(x, w, b)

            def mlp_act(x, w):
                return ops.swiglu(F.linear(x, w))
        if a.hidden_act != "silu":
            # GeGLU families: the projection, then the tanh-GELU gate
            def mlp_act(x, w, _proj=proj):
                g, u = _proj(x, w).chunk(2, dim=-1)
                return F.gelu(g.float(), approximate="tanh").to(g.dtype) * u
        x = F.embedding(ids, W["embed.weight"])
        if a.embed_scale:
            x = x * torch.tensor(a.embed_scale, dtype=x.dtype)
        resid = None
        T = ids.shape[0]
        for l in range(a.num_layers):
            pre = f"layers.{l}."
            h, r2 = ops.rms_norm(x, W[pre + "ln1"], a.rms_eps, residual=resid)
            resid = x if resid is None else r2
            qkv = proj(h, W[pre + "attn.qkv.weight"], W.get(pre + "attn.qkv.bias"))
            if a.qk_norm:
                q = qkv[:, : a.q_size].view(T, a.num_heads, a.head_dim)
                k = qkv[:, a.q_size: a.q_size + a.kv_size].view(T, a.num_kv_heads, a.head_dim)
                if qkv.is_cuda:
                    ops.ext().head_rmsnorm_(q, W[pre + "attn.q_norm"], a.rms_eps)
                    ops.ext().head_rmsnorm_(k, W[pre + "attn.k_norm"], a.rms_eps)
                else:
                    q.copy_(ops.head_rms_norm(q, W[pre + "attn.q_norm"], a.rms_eps))
                    k.copy_(ops.head_rms_norm(k, W[pre + "attn.k_norm"], a.rms_eps))
            if a.qk_norm_full:
                q = qkv[:, : a.q_size]
                k = qkv[:, a.q_size: a.q_size + a.kv_size]
                q.copy_(ops.rms_norm(q.contiguous(), W[pre + "attn.q_norm"], a.rms_eps)[0])
                k.copy_(ops.rms_norm(k.contiguous(), W[pre + "attn.k_norm"], a.rms_eps)[0])
            ops.rope_qkv_(qkv, pos, a.num_heads, a.num_kv_heads, a.head_dim, a.rope_spec,
                          k_cache=self.k_cache[l], v_cache=self.v_cache[l], slots=slots)
            q = qkv[:, : a.q_size].view(T, a.num_heads, a.head_dim)
            if mode == "prefill":
                o = ops.paged_prefill_attention(q, self.k_cache[l], self.v_cache[l], cu_q, kv_lens, block_table, max_q)
            else:
                o = ops.paged_decode_attention(q, self.k_cache[l], self.v_cache[l], block_table, kv_lens,
                                               splits=splits if self.is_cuda else None,
                                               scratch=self.decode_scratch if self.is_cuda else None)
            attn = proj(o.reshape(T, a.q_size), W[pre + "attn.o.weight"])
            if self.tp is not None:
                dist.all_reduce(attn, group=self.tp.group)
            h2, resid = ops.rms_norm(attn, W[pre + "ln2"], a.rms_eps, residual=resid)
            if a.is_moe:
                x = self._moe(h2, pre)
                if self.tp is not None:
                    dist.all_reduce(x, group=self.tp.group)
            else:
                x = proj(mlp_act(h2, W[pre + "mlp.gate_up.weight"]), W[pre + "mlp.down.weight"])
                if self.tp is not None:
                    dist.all_reduce(x, group=self.tp.group)
        hN, _ = ops.rms_norm(x, W["norm"], a.rms_eps, residual=resid)
        return hN

    def _moe(self, h, pre):
        y = self._moe_routed(h, pre)
        if self.args.shared_expert_intermediate_size:
            W = self.w
            sh = F.linear(ops.swiglu(F.linear(h, W[pre + "mlp.shared_gate_up.weight"])), W[pre + "mlp.shared_down.weight"])
            y = y + torch.sigmoid(F.linear(h, W[pre + "mlp.shared_gate.weight"]).float()).to(sh.dtype) * sh
        return y

    def _moe_routed_ep(self, h, pre):
        """Routed experts of a TP engine: top-k over all experts (identical on
        every rank), then only this rank's experts; entries routed elsewhere
        keep weight 0 (computed on local expert 0 and dropped by the combine),
        so the step has no host synchronisation."""
        from ..ops import moe as moe_ops
        from ..parallel.moe import moe_forward_local
        a, W = self.args, self.w
        w13, w2 = W[pre + "mlp.experts_w13"], W[pre + "mlp.experts_w2"]
        n_local = w13.shape[0]
        lo = self.tp.rank * n_local
        wt, ids, _ = moe_ops.route(F.linear(h, W[pre + "mlp.router.weight"]), W[pre + "mlp.router_prior"],
                                   a.num_experts_per_tok, bool(a.norm_topk_prob))
        ids = ids.long()
        local = (ids >= lo) & (ids < lo + n_local)
        wl = torch.where(local, wt, torch.zeros_like(wt))
        il = torch.where(local, ids - lo, torch.zeros_like(ids))
        if moe_ops.supported(h, w13, w2):
            return moe_ops.moe_mlp_routed(h, wl, il, w13, w2)
        return moe_forward_local(h, wl.to(h.dtype), il, w13, w2)

    def _moe_routed(self, h, pre):
        from ..ops import moe as moe_ops
        from ..parallel.moe import moe_forward_local
        if self.tp is not None and self.w[pre + "mlp.experts_w13"].shape[0] < self.args.num_experts:
            return self._moe_routed_ep(h, pre)
        # (a TP engine holding every expert at 1/P of its width, from a TP trainer's
        # shards, runs the plain path: its partial output joins the all-reduce)
        a, W = self.args, self.w
        if moe_ops.supported(h, W[pre + "mlp.experts_w13"], W[pre + "mlp.experts_w2"]):
            return moe_ops.moe_mlp(h, F.linear(h, W[pre + "mlp.router.weight"]).float(), W[pre + "mlp.router_prior"],
                                   W[pre + "mlp.experts_w13"], W[pre + "mlp.experts_w2"], a.num_experts_per_tok,
                                   bool(a.norm_topk_prob))
        logits = F.linear(h, W[pre + "mlp.router.weight"]).float() + W[pre + "mlp.router_prior"]
        probs = logits.softmax(-1)
        wt, idx = probs.topk(a.num_experts_per_tok, dim=-1)
        if a.norm_topk_prob:
            wt = wt / wt.sum(-1, keepdim=True)
        return moe_forward_local(h, wt.to(h.dtype), idx, W[pre + "mlp.experts_w13"], W[pre + "mlp.experts_w2"])

    # --------------------------------------------------------------- stats
    def engine_stats(self) -> dict:
        return {
            "num_waiting": len(self.waiting),
            "num_running": len(self.running),
            "kv_usage": self.bm.usage(),
            "version": self.version,
            "prefix_hit_rate": self.bm.hits / max(1, self.bm.queries),
            **self.stats,
        }
