"""Prompt sources and the data processor (C20).

Synthetic sources generate the workloads the benchmarks name:

* ``synthetic_tokens`` — random token-id prompts, lengths uniform in
  [prompt_len_min, prompt_len_max]; each trajectory gets a forced response
  length drawn from lognormal(mu, sigma) capped at ``response_len_cap``.
* ``addition`` — two-operand integer additions (operands uniform 0-999),
  char-level tokenised, padded to 16-32 tokens, answer after ``####``.

File datasets (``parquet`` / ``jsonl``, ``data.train_files``) use the
reference's row layout: ``prompt`` (chat messages or a string),
``data_source``, ``reward_model.ground_truth`` (or ``ground_truth`` /
``answer``) and ``extra_info``.  Prompts are rendered with the tokenizer's
chat template (``data.tokenizer``: an HF tokenizer directory; the byte-level
tokenizer with ChatML otherwise); rows longer than
``rollout.max_prompt_length`` are dropped at load time.  Each epoch visits
the rows in a fresh seeded permutation (file order with ``data.shuffle=false``).

``DataProcessor`` hands out prompt *groups* (``rollout_n`` samples share a
``uid`` / parent id), is seeded, and can save/load its cursor for resume
(reference: ``psrl/utils/dataset/data_processor.py:39``, ``sample_train_prompts`` :610).
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field

import numpy as np

# ---------------------------------------------------------------- tokenizer


class CharTokenizer:
    """Byte-level tokenizer: token = byte value + 3 (0 pad, 1 bos, 2 eos)."""

    pad_id, bos_id, eos_id = 0, 1, 2

    def __init__(self, vocab_size: int = 1024):
        assert vocab_size >= 259
        self.vocab_size = vocab_size

    def encode(self, s: str) -> list[int]:
        return [b + 3 for b in s.encode("utf-8")]

    def decode(self, ids) -> str:
        return bytes(i - 3 for i in ids if 3 <= i < 259).decode("utf-8", errors="replace")


@dataclass
class PromptItem:
    uid: int
    prompt_ids: list
    response_lens: list | None = None       # forced lengths per sample (synthetic)
    answer: int | None = None
    meta: dict = field(default_factory=dict)


class SyntheticTokenSource:
    def __init__(self, vocab_size: int, lo: int, hi: int, mu: float, sigma: float, cap: int, n: int, seed: int):
        self.vocab, self.lo, self.hi = vocab_size, lo, hi
        self.mu, self.sigma, self.cap, self.n = mu, sigma, cap, n
        self.seed = seed

    def item(self, uid: int) -> PromptItem:
        rng = np.random.default_rng([self.seed, uid])
        L = int(rng.integers(self.lo, self.hi + 1))
        ids = rng.integers(3, self.vocab, size=L).tolist()
        lens = np.minimum(np.maximum(1, rng.lognormal(self.mu, self.sigma, size=self.n)), self.cap).astype(int).tolist()
        return PromptItem(uid, ids, lens)


class AdditionSource:
    def __init__(self, tokenizer: CharTokenizer, seed: int):
        self.tok = tokenizer
        self.seed = seed
        self.vocab = tokenizer.vocab_size

    def item(self, uid: int) -> PromptItem:
        rng = random.Random(self.seed * 1_000_003 + uid)
        a, b = rng.randint(0, 999), rng.randint(0, 999)
        text = f"add {a}+{b}="
        target = rng.randint(16, 32)
        text = ("." * max(0, target - len(text) - 1)) + text
        ids = [self.tok.bos_id] + self.tok.encode(text)
        return PromptItem(uid, ids[:32], None, a + b)


class HFTokenizer:
    """Adapter giving an HF tokenizer the byte tokenizer's interface
    (``encode`` without special tokens, ``decode`` skipping them, ``eos_id``,
    ``vocab_size``) plus its own chat template."""

    def __init__(self, tok):
        self.tok = tok
        self.eos_id = tok.eos_token_id
        self.pad_id = tok.pad_token_id if tok.pad_token_id is not None else tok.eos_token_id
        self.bos_id = tok.bos_token_id
        self.vocab_size = len(tok)

    @classmethod
    def from_pretrained(cls, path: str) -> "HFTokenizer":
        from transformers import AutoTokenizer
        return cls(AutoTokenizer.from_pretrained(path))

    def encode(self, s: str) -> list[int]:
        return list(self.tok.encode(s, add_special_tokens=False))

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def apply_chat_template(self, messages, add_generation_prompt: bool = True, tokenize: bool = True):
        if getattr(self.tok, "chat_template", None):
            return self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                                tokenize=tokenize)
        from ..utils.common import chatml
        text = chatml(messages, add_generation_prompt)
        return self.encode(text) if tokenize else text


def _read_rows(path: str) -> list[dict]:
    if path.endswith(".parquet"):
        import pyarrow.parquet as pq
        return pq.read_table(path).to_pylist()
    import json
    with open(path) as fh:
        return [json.loads(line) for line in fh if line.strip()]


class FileSource:
    """Prompt rows from parquet / jsonl files (reference row layout)."""

    def __init__(self, files, tokenizer, max_prompt_len: int, seed: int, filter_overlong: bool = True,
                 shuffle: bool = True):
        from ..utils.common import apply_chat_template
        self.tok = tokenizer
        self.shuffle = bool(shuffle)
        self.seed = int(seed)
        self.vocab = getattr(tokenizer, "vocab_size", 1024)
        self.items: list[tuple[list[int], dict]] = []
        self.dropped = 0
        for f in ([files] if isinstance(files, str) else list(files)):
            for row in _read_rows(f):
                prompt = row.get("prompt")
                if isinstance(prompt, str):
                    prompt = [{"role": "user", "content": prompt}]
                ids = list(apply_chat_template(list(prompt), tokenizer))
                if len(ids) > max_prompt_len:
                    if filter_overlong:
                        self.dropped += 1
                        continue
                    ids = ids[-max_prompt_len:]
                rm = row.get("reward_model") or {}
                gt = rm.get("ground_truth") if isinstance(rm, dict) else None
                if gt is None:
                    gt = row.get("ground_truth", row.get("answer"))
                meta = {"data_source": row.get("data_source"), "ground_truth": gt,
                        "extra_info": row.get("extra_info") or {}}
                self.items.append((ids, meta))
        if not self.items:
            raise ValueError(f"no usable prompts in {files!r} ({self.dropped} longer than {max_prompt_len} tokens)")
        self._perm_epoch = -1
        self._perm: list[int] = []

    def item(self, uid: int) -> PromptItem:
        n = len(self.items)
        if uid >= (1 << 40):                      # validation uids: rows in file order
            ids, meta = self.items[(uid - (1 << 40)) % n]
            return PromptItem(uid, list(ids), None, None, dict(meta))
        epoch, k = divmod(int(uid), n)
        if epoch != self._perm_epoch:
            self._perm = (np.random.default_rng([self.seed, epoch]).permutation(n).tolist() if self.shuffle
                          else list(range(n)))
            self._perm_epoch = epoch
        ids, meta = self.items[self._perm[k]]
        return PromptItem(uid, list(ids), None, None, dict(meta))


class DataProcessor:
    """Seeded stream of prompt groups; cursor is checkpointable."""

    def __init__(self, cfg, vocab_size: int, rollout_n: int, tokenizer: CharTokenizer | None = None):
        d = cfg.data
        self.kind = d.kind
        self.rollout_n = rollout_n
        if tokenizer is None and d.get("tokenizer"):
            tokenizer = HFTokenizer.from_pretrained(str(d.tokenizer))
        self.tokenizer = tokenizer or CharTokenizer(max(259, min(vocab_size, 1024)))
        if d.kind == "synthetic_tokens":
            self.src = SyntheticTokenSource(vocab_size, int(d.prompt_len_min), int(d.prompt_len_max),
                                            float(d.response_len_mu), float(d.response_len_sigma),
                                            int(d.response_len_cap), rollout_n, int(d.seed))
        elif d.kind == "addition":
            self.src = AdditionSource(self.tokenizer, int(d.seed))
        elif d.kind in ("parquet", "jsonl", "files"):
            self.src = FileSource(d.train_files, self.tokenizer, int(cfg.rollout.max_prompt_length), int(d.seed),
                                  bool(d.get("filter_overlong_prompts", True)), bool(d.get("shuffle", True)))
            if d.get("val_files"):
                self.val_src = FileSource(d.val_files, self.tokenizer, int(cfg.rollout.max_prompt_length),
                                          int(d.seed), bool(d.get("filter_overlong_prompts", True)))
        else:
            raise ValueError(f"unsupported data.kind {d.kind!r} (synthetic_tokens|addition|parquet|jsonl)")
        self.cursor = 0

    def next_group(self) -> PromptItem:
        it = self.src.item(self.cursor)
        self.cursor += 1
        return it

    # validation prompts come from their own uid range, disjoint from training
    VAL_UID_BASE = 1 << 40

    def validation_items(self, n: int) -> list[PromptItem]:
        """The first ``n`` validation prompts (deterministic, never trained on)."""
        src = getattr(self, "val_src", None) or self.src
        return [src.item(self.VAL_UID_BASE + i) for i in range(int(n))]

    def state_dict(self) -> dict:
        return {"cursor": self.cursor}

    def load_state_dict(self, st: dict) -> None:
        self.cursor = int(st["cursor"])
