"""Token caches in the TreeCache layout the reference trains from.

A reference cache split (megagpt-speedrun/data.py:119-165, 296-330) is a directory holding
``shard_ledger.json`` (``is_finished: true`` once complete) and one directory per field --
``input_ids/``, and ``assistant_masks/`` for chat data -- each a jagged array: a flat ``data``
array of every row's values back to back and an ``offsets`` array of row ends, both zarr arrays
(``utils.zarr_io``). ``offsets`` holds the row count in entry 0 and the end of row i in entry
i + 1; a plain ``[0, end_0, end_1, ...]`` offsets array (first entry 0) reads the same way.

``write_tree_cache`` writes that layout, ``TreeCache`` reads it row by row, and
``to_native_cache`` turns its ``input_ids`` (and ``assistant_masks`` as per-token loss masks)
into the native loader's shards (``data.tokenize``), so a reference cache trains here without
re-tokenizing.
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterable

import numpy as np

from ..utils import zarr_io

LEDGER = "shard_ledger.json"


def write_tree_cache(root: str, rows: Iterable[dict[str, np.ndarray]], fields: tuple[str, ...] = ("input_ids",),
                     *, dtypes: dict[str, str] | None = None, zstd: bool = True) -> dict:
    """Write ``rows`` (each a dict of 1-D arrays, one per field) as a finished TreeCache at ``root``."""
    dtypes = dict(dtypes or {})
    vals = {f: [] for f in fields}
    ends = {f: [] for f in fields}
    n = 0
    for row in rows:
        for f in fields:
            a = np.asarray(row[f]).reshape(-1)
            vals[f].append(a)
            ends[f].append((ends[f][-1] if ends[f] else 0) + len(a))
        n += 1
    os.makedirs(root, exist_ok=True)
    for f in fields:
        dt = dtypes.get(f, "int32" if f == "input_ids" else None)
        data = np.concatenate(vals[f]) if vals[f] else np.zeros(0, dtype=np.int32)
        if dt is not None:
            data = data.astype(dt)
        offsets = np.asarray([n] + ends[f], dtype=np.int64)
        zarr_io.write_array(os.path.join(root, f, "data"), data, zstd=zstd)
        zarr_io.write_array(os.path.join(root, f, "offsets"), offsets, zstd=zstd)
    ledger = {"total_num_rows": n, "is_finished": True, "fields": list(fields),
              "field_counts": {f: int(ends[f][-1]) if ends[f] else 0 for f in fields}}
    with open(os.path.join(root, LEDGER), "w") as fh:
        json.dump(ledger, fh, indent=1)
    return ledger


class TreeCache:
    """Row access to a finished TreeCache split (every field's arrays are read once, eagerly)."""

    def __init__(self, root: str):
        lp = os.path.join(root, LEDGER)
        if not os.path.exists(lp):
            raise FileNotFoundError(f"{root}: no {LEDGER} (not a TreeCache split)")
        with open(lp) as fh:
            self.ledger = json.load(fh)
        if not self.ledger.get("is_finished", False):
            raise ValueError(f"{root}: cache is not finished (is_finished is false)")
        self.root = root
        self.fields = [d for d in sorted(os.listdir(root))
                       if zarr_io.is_array(os.path.join(root, d, "data"))
                       and zarr_io.is_array(os.path.join(root, d, "offsets"))]
        if not self.fields:
            raise ValueError(f"{root}: no jagged-array fields")
        self._data, self._starts = {}, {}
        for f in self.fields:
            data = zarr_io.read_array(os.path.join(root, f, "data")).reshape(-1)
            off = zarr_io.read_array(os.path.join(root, f, "offsets")).astype(np.int64).reshape(-1)
            if len(off) and off[0] != 0:  # count-prefixed: [n, end_0, ..., end_{n-1}]
                n = int(off[0])
                ends = off[1: n + 1]
            else:  # plain: [0, end_0, ...]
                ends = off[1:]
            self._starts[f] = np.concatenate([[0], ends]).astype(np.int64)
            self._data[f] = data
        self._n = len(self._starts[self.fields[0]]) - 1

    def __len__(self) -> int:
        return self._n

    def __getitem__(self, i: int) -> dict[str, np.ndarray]:
        if not 0 <= i < self._n:
            raise IndexError(i)
        return {f: self._data[f][self._starts[f][i]: self._starts[f][i + 1]] for f in self.fields}

    def field(self, name: str) -> tuple[np.ndarray, np.ndarray]:
        """(values, row starts with a final end) of one field."""
        return self._data[name], self._starts[name]


def to_native_cache(root: str, cache_path: str, *, eos_id: int | None = None, vocab_size: int | None = None,
                    shard_tokens: int = 1 << 28) -> dict:
    """Convert a TreeCache split's ``input_ids`` rows (one document each, end-of-document token
    already included by the reference's tokenizer) into native loader shards; ``assistant_masks``,
    when present, become the shards' per-token loss masks."""
    tc = TreeCache(root)
    if "input_ids" not in tc.fields:
        raise ValueError(f"{root}: no input_ids field")
    ids, starts = tc.field("input_ids")
    masks = tc.field("assistant_masks")[0] if "assistant_masks" in tc.fields else None
    os.makedirs(cache_path, exist_ok=True)
    shards = []
    r0 = 0
    n_rows = len(tc)
    while r0 < n_rows:
        t0 = starts[r0]
        r1 = int(np.searchsorted(starts, t0 + shard_tokens, side="right")) - 1
        r1 = min(max(r1, r0 + 1), n_rows)
        t1 = starts[r1]
        i = len(shards)
        names = {"tokens": f"tokens-{i:05d}.bin", "docs": f"docs-{i:05d}.bin"}
        ids[t0:t1].astype("<u4").tofile(os.path.join(cache_path, names["tokens"]))
        (starts[r0 + 1: r1 + 1] - t0).astype("<u8").tofile(os.path.join(cache_path, names["docs"]))
        if masks is not None:
            names["mask"] = f"mask-{i:05d}.bin"
            (masks[t0:t1] != 0).astype(np.uint8).tofile(os.path.join(cache_path, names["mask"]))
        shards.append({**names, "num_tokens": int(t1 - t0), "num_docs": int(r1 - r0)})
        r0 = r1
    meta = {"shards": shards, "num_tokens": int(starts[-1]), "num_docs": n_rows, "source": "treecache:" + root,
            "vocab_size": vocab_size if vocab_size is not None else int(ids.max()) + 1 if len(ids) else 0,
            "eos_id": eos_id}
    if masks is not None:
        meta["format"] = "chat"
    with open(os.path.join(cache_path, "meta.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    with open(os.path.join(cache_path, ".success"), "w") as fh:
        fh.write("ok\n")
    return meta
