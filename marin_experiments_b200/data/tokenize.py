"""Tokenize step: text documents -> token cache (the marin ``tokenize`` step the tiny-stories
template runs before training, tiny-stories/launch.py:141-153, with its ``sample_count`` cap).

Input: ``.jsonl`` files (one JSON object per line, text under ``text_key``) or plain ``.txt`` files
(one document per file, or one per line with ``line_docs``). Output directory:

* ``tokens-NNNNN.bin``: little-endian uint32 token ids of the concatenated documents, each followed
  by the tokenizer's end-of-document id;
* ``docs-NNNNN.bin``: little-endian uint64 end offsets of the documents within the shard;
* ``meta.json``: shard list, token/doc counts, tokenizer name and vocabulary size;
* ``.success``: written last, so an interrupted step is redone.

Tokenizers: a local Hugging Face ``tokenizer.json`` (``tokenizers`` library; there is no network)
or the built-in ``"bytes"`` tokenizer (ids 0-255 are bytes, 256 is end-of-document).
"""

from __future__ import annotations

import glob
import json
import os
from collections.abc import Iterable, Iterator
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class TokenizeConfig:
    train_paths: tuple[str, ...]
    cache_path: str
    tokenizer: str = "bytes"
    text_key: str = "text"
    sample_count: int | None = None
    shard_tokens: int = 1 << 28
    line_docs: bool = False
    prepend_bos: bool = False  # start every document with the tokenizer's begin-of-sequence token


class ByteTokenizer:
    vocab_size = 257
    eos_id = 256
    name = "bytes"

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Iterable[int]) -> str:
        return bytes(i for i in ids if i < 256).decode("utf-8", errors="replace")


class HFTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer

        self.tok = Tokenizer.from_file(path)
        self.name = path
        self.vocab_size = self.tok.get_vocab_size()
        eos = None
        for cand in ("<|endoftext|>", "</s>", "<|end_of_text|>", "<eos>", "<|eos|>"):
            eos = self.tok.token_to_id(cand)
            if eos is not None:
                break
        self.eos_id = eos if eos is not None else self.vocab_size - 1
        self.bos_id = None
        for cand in ("<|begin_of_text|>", "<s>", "<bos>", "<|bos|>"):
            self.bos_id = self.tok.token_to_id(cand)
            if self.bos_id is not None:
                break

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False).ids

    def decode(self, ids: Iterable[int]) -> str:
        return self.tok.decode(list(ids))


def load_tokenizer(name: str):
    """``bytes``, a ``tokenizer.json`` path or a directory holding one, or ``trained/<name>``: a
    tokenizer this project trained, from the mirror under ``MXK_TOKENIZER_MIRROR``."""
    if name == "bytes":
        return ByteTokenizer()
    if name.startswith("trained/") and not os.path.exists(name):
        mirror = os.environ.get("MXK_TOKENIZER_MIRROR", "")
        if not mirror:
            raise FileNotFoundError(f"tokenizer {name!r}: set MXK_TOKENIZER_MIRROR to the trained-tokenizer mirror")
        name = os.path.join(mirror, "tokenizers", name)
    path = name if name.endswith(".json") else os.path.join(name, "tokenizer.json")
    if not os.path.exists(path):
        raise FileNotFoundError(f"tokenizer {name!r}: no local tokenizer.json (no network access)")
    return HFTokenizer(path)


def _expand(paths: Iterable[str]) -> list[str]:
    out = []
    for p in paths:
        if os.path.isdir(p):
            out += sorted(glob.glob(os.path.join(p, "**", "*.jsonl"), recursive=True))
            out += sorted(glob.glob(os.path.join(p, "**", "*.txt"), recursive=True))
        else:
            out += sorted(glob.glob(p)) or [p]
    return out


def iter_documents(cfg: TokenizeConfig) -> Iterator[str]:
    n = 0
    for path in _expand(cfg.train_paths):
        if path.endswith(".jsonl"):
            with open(path) as f:
                for line in f:
                    line = line.strip()
                    if not line:
                        continue
                    yield json.loads(line)[cfg.text_key]
                    n += 1
                    if cfg.sample_count is not None and n >= cfg.sample_count:
                        return
        else:
            with open(path, encoding="utf-8") as f:
                docs = f.read().splitlines() if cfg.line_docs else [f.read()]
            for d in docs:
                if d:
                    yield d
                    n += 1
                    if cfg.sample_count is not None and n >= cfg.sample_count:
                        return


def is_complete(cache_path: str) -> bool:
    return os.path.exists(os.path.join(cache_path, ".success"))


def tokenize(cfg: TokenizeConfig) -> dict:
    """Run the step (a no-op when ``cache_path`` already holds a complete cache)."""
    if is_complete(cfg.cache_path):
        with open(os.path.join(cfg.cache_path, "meta.json")) as f:
            return json.load(f)
    os.makedirs(cfg.cache_path, exist_ok=True)
    tok = load_tokenizer(cfg.tokenizer)
    if tok.vocab_size >= 1 << 32:
        raise ValueError("vocabulary does not fit uint32 ids")
    shards, buf, ends = [], [], []
    n_tok = n_docs = 0
    shard_len = 0

    def flush():
        nonlocal buf, ends, shard_len
        if not ends:
            return
        i = len(shards)
        tname, dname = f"tokens-{i:05d}.bin", f"docs-{i:05d}.bin"
        np.concatenate(buf).astype("<u4").tofile(os.path.join(cfg.cache_path, tname))
        np.asarray(ends, dtype="<u8").tofile(os.path.join(cfg.cache_path, dname))
        shards.append({"tokens": tname, "docs": dname, "num_tokens": int(shard_len), "num_docs": len(ends)})
        buf, ends, shard_len = [], [], 0

    bos = [tok.bos_id] if cfg.prepend_bos and getattr(tok, "bos_id", None) is not None else []
    for text in iter_documents(cfg):
        ids = np.asarray(bos + tok.encode(text) + [tok.eos_id], dtype=np.uint32)
        buf.append(ids)
        shard_len += len(ids)
        ends.append(shard_len)
        n_tok += len(ids)
        n_docs += 1
        if shard_len >= cfg.shard_tokens:
            flush()
    flush()
    if not shards:
        raise ValueError(f"no documents found under {cfg.train_paths}")
    meta = {"shards": shards, "num_tokens": n_tok, "num_docs": n_docs, "tokenizer": tok.name,
            "vocab_size": tok.vocab_size, "eos_id": tok.eos_id}
    with open(os.path.join(cfg.cache_path, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    with open(os.path.join(cfg.cache_path, ".success"), "w") as f:
        f.write("ok\n")
    return meta
