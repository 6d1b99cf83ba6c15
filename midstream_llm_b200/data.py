"""Synthetic token batches standing in for the (absent) Jishui corpus.

Token ids are drawn i.i.d. with p(i) ∝ (i+1)^-s (Zipf, s = 1.1) over the
vocabulary from a numpy Generator seeded per stream (per rank for data
parallel runs), in [batch, seq+1] rows; inputs are row[:, :-1] and targets
row[:, 1:], as `tensor_batch` splits packed rows in the reference trainer
(Midstream-LLM src/jishui/pretrain_torch.py:38-40).
"""
from __future__ import annotations

import numpy as np
import torch


class ZipfBatches:
    """Deterministic stream of [batch, seq+1] int64 token rows."""

    def __init__(self, vocab: int, batch: int, seq: int, seed: int, s: float = 1.1):
        w = (np.arange(vocab, dtype=np.float64) + 1.0) ** (-s)
        self.p = w / w.sum()
        self.vocab, self.batch, self.seq, self.seed = vocab, batch, seq, seed
        self.rng = np.random.default_rng(seed)
        self.emitted = 0

    def next_rows(self) -> np.ndarray:
        self.emitted += 1
        return self.rng.choice(self.vocab, size=(self.batch, self.seq + 1), p=self.p).astype(np.int64)

    def state_dict(self) -> dict:
        return {"batches_emitted": self.emitted, "rng_state": self.rng.bit_generator.state}

    def load_state_dict(self, state: dict) -> None:
        self.emitted = int(state["batches_emitted"])
        self.rng.bit_generator.state = state["rng_state"]


def tensor_batch(rows: np.ndarray, device, pinned: bool = True):
    """(inputs, targets) on `device` from [B, T+1] integer rows (any integer dtype, widened to int64 as
    pretrain_torch.py:38-40 does)."""
    t = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.int64))
    if pinned and torch.device(device).type == "cuda":
        t = t.pin_memory()
    t = t.to(device, non_blocking=True)
    return t[:, :-1], t[:, 1:]
