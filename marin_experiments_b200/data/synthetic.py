"""Synthetic token data.

``SyntheticGrugDataset`` reproduces megagpt-speedrun/synth_data.py:25-70: example ``i`` is a
deterministic function of ``i`` (tokens uniform in ``[1, vocab)``), with packed-document segment ids
``arange(seq) // doc_len``. ``UniformTokenBatches`` draws whole batches of uniform ids in
``[0, vocab)`` from one seeded generator (the benchmark configurations' "uniform-random token ids
(seed s)"). Both return host tensors; ``pin=True`` gives page-locked memory for async copies.
"""

from __future__ import annotations

import numpy as np
import torch


class SyntheticGrugDataset:
    def __init__(self, seq_len: int, vocab_size: int, doc_len: int = 1024, seed: int = 0):
        self.seq_len, self.vocab_size, self.seed = int(seq_len), int(vocab_size), int(seed)
        chunk = max(1, min(int(doc_len), self.seq_len))
        self.segment_ids = torch.from_numpy((np.arange(self.seq_len) // chunk).astype(np.int32))

    def __len__(self) -> int:
        return 1 << 31

    def example(self, idx: int) -> np.ndarray:
        rng = np.random.default_rng((int(idx) + (self.seed << 32)) & 0x7FFFFFFFFFFFFFFF)
        return rng.integers(1, self.vocab_size, size=self.seq_len, dtype=np.int64)

    def batch(self, indices, pin: bool = False) -> dict[str, torch.Tensor]:
        toks = np.stack([self.example(i) for i in indices])
        t = torch.from_numpy(toks)
        seg = self.segment_ids.unsqueeze(0).expand(len(indices), -1).contiguous()
        if pin:
            t, seg = t.pin_memory(), seg.pin_memory()
        return {"tokens": t, "segment_ids": seg}


class UniformTokenBatches:
    """Iterator of ``{"tokens": [batch, seq] int64}`` with ids uniform in ``[0, vocab)``."""

    def __init__(self, batch: int, seq_len: int, vocab_size: int, seed: int = 0, pin: bool = False,
                 rank: int = 0):
        self.batch, self.seq_len, self.vocab_size, self.pin = batch, seq_len, vocab_size, pin
        self.gen = torch.Generator().manual_seed(seed * 1_000_003 + rank)

    def __iter__(self):
        return self

    def __next__(self) -> dict[str, torch.Tensor]:
        t = torch.randint(0, self.vocab_size, (self.batch, self.seq_len), generator=self.gen)
        if self.pin:
            t = t.pin_memory()
        return {"tokens": t}
