"""Data pipeline front end over the native runtime (``_mxrt``).

* ``build_dataset(cfg, seq_len, vocab)`` turns a ``DataConfig`` into a native dataset:
  ``synthetic`` (deterministic per-index random ids in ``[1, vocab)`` with packed ``doc_len``
  segments, megagpt-speedrun/synth_data.py:25-70), ``cache`` (a token cache written by
  ``data.tokenize``), or ``mixture`` (weighted caches). Every dataset is served through a block
  mixture, as the reference wraps even its synthetic source in a one-component ``MixtureDataset``
  (megagpt-speedrun/train.py:110-143, megagpt-speedrun/synth_data.py:57-70).
* ``DataLoader`` yields this rank's slice of each global batch (``tokens``, ``segment_ids``,
  ``loss_weight``) from page-locked host buffers filled ahead of time by native threads
  (megagpt-speedrun/train.py:149-172 keeps 128 batches buffered; here ``depth`` slots). A slot is
  recycled only after the CUDA work enqueued after it was handed out (its host-to-device copy)
  has completed, so non-blocking copies never read a buffer that is being refilled.

Example ``i`` of step ``s`` on rank ``r`` is global example ``s * global_batch + r * local_batch + i``;
the stream is a pure function of (config, seed, step), so a resumed run sees the same batches.
"""

from __future__ import annotations

import json
import os
from collections import deque

import torch

from ..runtime import rt

STOP = {"restart": 0, "first_exhausted": 1}


def open_cache(cache_dir: str, seq_len: int, seed: int, shuffle: bool = True):
    """Native ``TokenSeqDataset`` over a cache directory written by ``data.tokenize``."""
    with open(os.path.join(cache_dir, "meta.json")) as f:
        meta = json.load(f)
    toks = [os.path.join(cache_dir, s["tokens"]) for s in meta["shards"]]
    docs = [os.path.join(cache_dir, s["docs"]) for s in meta["shards"]]
    masks = [os.path.join(cache_dir, s["mask"]) for s in meta["shards"]] if all("mask" in s for s in meta["shards"]) \
        else []
    return rt().TokenSeqDataset(toks, docs, seq_len, seed, shuffle, masks)


def build_dataset(cfg, seq_len: int, vocab_size: int, *, block_size: int = 2048, stop_strategy: str = "restart"):
    m = rt()
    seed = int(cfg.seed)
    if cfg.source == "remote":
        from .remote import MIXES, data_config

        if cfg.mix not in MIXES:
            raise ValueError(f"unknown remote mixture {cfg.mix!r}; one of {sorted(MIXES)}")
        cfg = data_config(MIXES[cfg.mix], cfg.cache_dir or os.environ.get("MXK_DATA_ROOT", "data_cache"), seed=seed)
    if cfg.source in ("synthetic", "uniform"):
        comps = [m.SyntheticDataset(seq_len, vocab_size, cfg.doc_len if cfg.source == "synthetic" else seq_len, seed)]
        weights = [[1.0]]
    elif cfg.source == "cache":
        comps = [open_cache(cfg.cache_dir, seq_len, seed)]
        weights = [[1.0]]
    elif cfg.source == "mixture":
        if not cfg.components:
            raise ValueError("mixture data needs components (name, cache_dir, weight)")
        comps = [open_cache(d, seq_len, seed + i) for i, (_, d, _) in enumerate(cfg.components)]
        weights = [[float(w) for (_, _, w) in cfg.components]]
    else:
        raise ValueError(f"unknown data source {cfg.source}")
    return m.MixtureDataset(comps, [0], weights, block_size, seed, STOP[stop_strategy])


def mixture_weights_at(stages: list[tuple[int, dict[str, float]]], step: int) -> dict[str, float]:
    """Weights in force at ``step`` for a staged mixture ``[(start_step, {name: w}), ...]``
    (the per-stage weights the reference logs, megagpt-speedrun/train.py:253-270)."""
    cur = stages[0][1]
    for start, w in stages:
        if start <= step:
            cur = w
    return cur


class DataLoader:
    def __init__(self, dataset, global_batch: int, *, rank: int = 0, world: int = 1, start_step: int = 0,
                 depth: int = 4, threads: int = 4, pin: bool | None = None, timeout_s: float = 600.0):
        if global_batch % world:
            raise ValueError(f"global batch {global_batch} not divisible by {world} ranks")
        self.ds = dataset
        self.local = global_batch // world
        self.seq_len = dataset.seq_len()
        pin = torch.cuda.is_available() if pin is None else pin
        shape = (self.local, self.seq_len)
        mk = (lambda dt: torch.empty(shape, dtype=dt).pin_memory()) if pin else (lambda dt: torch.empty(shape, dtype=dt))
        self.slots = [(mk(torch.int32), mk(torch.int32), mk(torch.float32)) for _ in range(depth)]
        self._pf = rt().Prefetcher(dataset, self.local, global_batch, rank, start_step,
                                   [s[0] for s in self.slots], [s[1] for s in self.slots],
                                   [s[2] for s in self.slots], threads)
        self.timeout_s = timeout_s
        self._out: deque = deque()  # (slot, cuda event or None) handed out, not yet recycled
        self.step = start_step

    def __iter__(self):
        return self

    def _recycle(self, force_one: bool) -> None:
        while self._out:
            slot, ev = self._out[0]
            if ev is not None and not ev.query():
                if not force_one:
                    return
                ev.synchronize()
            self._out.popleft()
            self._pf.release(slot)
            force_one = False

    def __next__(self) -> dict[str, torch.Tensor]:
        if self._out and self._out[-1][1] is None and torch.cuda.is_available():
            ev = torch.cuda.Event()
            ev.record()  # after the consumer's copy of the previous batch
            self._out[-1] = (self._out[-1][0], ev)
        elif self._out and not torch.cuda.is_available():
            self._out[-1] = (self._out[-1][0], None)
        self._recycle(force_one=len(self._out) >= len(self.slots) - 1)
        try:
            slot, step = self._pf.next(self.timeout_s)
        except IndexError as e:  # std::out_of_range: a component ran out under first_exhausted
            raise StopIteration from e
        self._out.append((slot, None))
        self.step = step + 1
        tok, seg, lw = self.slots[slot]
        return {"tokens": tok, "segment_ids": seg, "loss_weight": lw}
