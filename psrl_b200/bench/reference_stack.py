"""The reference's library stack, measured piece by piece on this machine.

The reference cannot run end to end here (Ray, veRL, Hydra, NIXL and its
gateway have no offline wheels), so its two hot loops are timed with the
libraries it runs them on, at the shapes of the 3B DAPO recipe:

* ``rollout``: vLLM (the reference pins ``releases/v0.22.0``,
  ``scripts/install_basic.sh:104``) generating forced-length responses from a
  random-init Qwen2.5-3B-shaped model (``load_format="dummy"``), reported as
  generated tokens/s;
* ``train``: one micro-batch forward + backward of the HF transformers
  Qwen2 model with flash-attention 2 (veRL's FSDP engine on one GPU), reported
  as trained tokens/s;
* ``nccl``: all-reduce / all-gather / reduce-scatter bus bandwidth
  (``psrl_b200.bench.comm_bench`` measures the same collectives for this
  framework).

Each case prints one JSON line; the matching numbers of this framework come
from ``psrl_b200.bench.rollout_bench`` and ``psrl_b200.bench.kernel_bench --only train_mb``.

    python -m psrl_b200.bench.reference_stack --case rollout --num-requests 256 --prompt-len 256 --output-len 512
    python -m psrl_b200.bench.reference_stack --case train
"""

from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import torch

QWEN25_3B = dict(architectures=["Qwen2ForCausalLM"], model_type="qwen2", vocab_size=151936, hidden_size=2048,
                 intermediate_size=11008, num_hidden_layers=36, num_attention_heads=16, num_key_value_heads=2,
                 max_position_embeddings=32768, rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=True,
                 torch_dtype="bfloat16", hidden_act="silu", bos_token_id=151643, eos_token_id=151643,
                 sliding_window=None, use_sliding_window=False, attention_dropout=0.0)


def _config_dir() -> str:
    d = tempfile.mkdtemp(prefix="qwen25_3b_cfg_")
    with open(os.path.join(d, "config.json"), "w") as fh:
        json.dump(QWEN25_3B, fh)
    return d


def bench_rollout(args) -> dict:
    from vllm import LLM, SamplingParams
    llm = LLM(model=_config_dir(), load_format="dummy", dtype="bfloat16", skip_tokenizer_init=True,
              gpu_memory_utilization=0.85, max_num_seqs=args.max_num_seqs,
              max_model_len=args.prompt_len + args.output_len + 16, enable_prefix_caching=False, seed=0)
    g = torch.Generator().manual_seed(0)
    prompts = [{"prompt_token_ids": torch.randint(3, 151000, (args.prompt_len,), generator=g).tolist()}
               for _ in range(args.num_requests)]
    sp = SamplingParams(max_tokens=args.output_len, ignore_eos=True, temperature=1.0, seed=0)
    llm.generate(prompts[: min(32, len(prompts))], sp, use_tqdm=False)      # warm-up (graphs, allocator)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    outs = llm.generate(prompts, sp, use_tqdm=False)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    n = sum(len(o.outputs[0].token_ids) for o in outs)
    return {"case": "reference-stack rollout (vLLM 0.22, Qwen2.5-3B shape, dummy weights)",
            "num_requests": args.num_requests, "prompt_len": args.prompt_len, "output_len": args.output_len,
            "max_num_seqs": args.max_num_seqs, "generated_tokens": n, "wall_s": round(wall, 3),
            "gen_tok_per_s": round(n / wall, 1)}


def bench_train(args) -> dict:
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(**{k: v for k, v in QWEN25_3B.items() if k not in ("architectures", "torch_dtype")})
    cfg._attn_implementation = "flash_attention_2"
    with torch.device("cuda"):
        model = Qwen2ForCausalLM(cfg).to(torch.bfloat16)
    model.gradient_checkpointing_disable()
    L, nseq = args.seq_len, args.num_seqs
    ids = torch.randint(3, 151000, (1, L * nseq), device="cuda")
    pos = torch.arange(L, device="cuda").repeat(nseq)[None]          # packed sequences (flash-attn varlen)

    def step():
        out = model(input_ids=ids, position_ids=pos, labels=ids)
        out.loss.backward()
        model.zero_grad(set_to_none=True)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.iters):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.iters
    return {"case": "reference-stack train micro-batch (HF Qwen2 + flash-attn 2 + cuBLAS, Qwen2.5-3B shape)",
            "tokens": L * nseq, "ms": round(ms, 2), "tok_per_s": round(L * nseq / (ms / 1e3), 1)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=["rollout", "train"], required=True)
    ap.add_argument("--num-requests", type=int, default=256)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--prompt-len", type=int, default=256)
    ap.add_argument("--output-len", type=int, default=512)
    ap.add_argument("--seq-len", type=int, default=1700)
    ap.add_argument("--num-seqs", type=int, default=6)
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args()
    res = bench_rollout(args) if args.case == "rollout" else bench_train(args)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
