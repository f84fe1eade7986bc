"""Prompt sources and the data processor (C20).

Synthetic sources generate the workloads the benchmarks name:

* ``synthetic_tokens`` — random token-id prompts, lengths uniform in
  [prompt_len_min, prompt_len_max]; each trajectory gets a forced response
  length drawn from lognormal(mu, sigma) capped at ``response_len_cap``.
* ``addition`` — two-operand integer additions (operands uniform 0-999),
  char-level tokenised, padded to 16-32 tokens, answer after ``####``.

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


class DataProcessor:
    """Seeded stream of prompt groups; cursor is checkpointable."""

    def __init__(self, cfg, vocab_size: int, rollout_n: int, tokenizer: CharTokenizer | None = None):
        d = cfg.data
        self.kind = d.kind
        self.rollout_n = rollout_n
        self.tokenizer = tokenizer or CharTokenizer(max(259, min(vocab_size, 1024)))
        if d.kind == "synthetic_tokens":
            self.src = SyntheticTokenSource(vocab_size, int(d.prompt_len_min), int(d.prompt_len_max),
                                            float(d.response_len_mu), float(d.response_len_sigma),
                                            int(d.response_len_cap), rollout_n, int(d.seed))
        elif d.kind == "addition":
            self.src = AdditionSource(self.tokenizer, int(d.seed))
        else:
            raise ValueError(f"unsupported data.kind {d.kind!r} (synthetic_tokens|addition)")
        self.cursor = 0

    def next_group(self) -> PromptItem:
        it = self.src.item(self.cursor)
        self.cursor += 1
        return it

    # validation prompts come from their own uid range, disjoint from training
    VAL_UID_BASE = 1 << 40

    def validation_items(self, n: int) -> list[PromptItem]:
        """The first ``n`` validation prompts (deterministic, never trained on)."""
        return [self.src.item(self.VAL_UID_BASE + i) for i in range(int(n))]

    def state_dict(self) -> dict:
        return {"cursor": self.cursor}

    def load_state_dict(self, st: dict) -> None:
        self.cursor = int(st["cursor"])
