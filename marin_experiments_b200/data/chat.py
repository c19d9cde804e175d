"""Chat (SFT) data: ChatML rendering, assistant-only loss masks and a chat token cache
(megagpt-speedrun/data.py:244-351 ``ChatLmDatasetFormat(mask_user_turns=True)``;
openthoughts-agent/training/agent_sft.py:39-307).

A conversation renders as ``<|im_start|>{role}\\n{content}<|im_end|>\\n`` per message. The loss mask is
1 on every assistant turn's ``{content}<|im_end|>\\n`` (what the model must produce) and 0 on system /
user / tool turns and on the role headers. ``write_chat_cache`` tokenizes a JSONL of
``{"messages": [{"role", "content"}, ...]}`` into the token-cache format of ``data.tokenize`` plus one
uint8 mask file per shard, which the native loader turns into next-token loss weights.
"""

from __future__ import annotations

import json
import os
from collections.abc import Iterable

import numpy as np

IM_START, IM_END = "<|im_start|>", "<|im_end|>"


def render_chatml(messages: list[dict], add_generation_prompt: bool = False) -> str:
    parts = [f"{IM_START}{m['role']}\n{m['content']}{IM_END}\n" for m in messages]
    if add_generation_prompt:
        parts.append(f"{IM_START}assistant\n")
    return "".join(parts)


def _special_id(tok, text: str):
    inner = getattr(tok, "tok", None)
    if inner is not None:
        return inner.token_to_id(text)
    return None


def encode_chat(messages: list[dict], tok) -> tuple[list[int], list[int]]:
    """``(ids, mask)`` with mask 1 on assistant content + end marker + newline."""
    ids, mask = [], []

    def add(text: str, m: int):
        t = tok.encode(text)
        ids.extend(t)
        mask.extend([m] * len(t))

    s_id, e_id = _special_id(tok, IM_START), _special_id(tok, IM_END)
    for msg in messages:
        train = 1 if msg["role"] == "assistant" else 0
        if s_id is not None:
            ids.append(s_id)
            mask.append(0)
            add(f"{msg['role']}\n", 0)
        else:
            add(f"{IM_START}{msg['role']}\n", 0)
        add(msg["content"], train)
        if e_id is not None:
            ids.append(e_id)
            mask.append(train)
        else:
            add(IM_END, train)
        add("\n", train)
    return ids, mask


def write_chat_cache(jsonl_paths: Iterable[str], cache_path: str, tok, messages_key: str = "messages",
                     shard_tokens: int = 1 << 28) -> dict:
    os.makedirs(cache_path, exist_ok=True)
    shards, toks, masks, ends = [], [], [], []
    total = n_docs = cur = 0

    def flush():
        nonlocal toks, masks, ends, cur
        if not ends:
            return
        i = len(shards)
        names = {"tokens": f"tokens-{i:05d}.bin", "docs": f"docs-{i:05d}.bin", "mask": f"mask-{i:05d}.bin"}
        np.concatenate(toks).astype("<u4").tofile(os.path.join(cache_path, names["tokens"]))
        np.asarray(ends, dtype="<u8").tofile(os.path.join(cache_path, names["docs"]))
        np.concatenate(masks).astype(np.uint8).tofile(os.path.join(cache_path, names["mask"]))
        shards.append({**names, "num_tokens": int(cur), "num_docs": len(ends)})
        toks, masks, ends, cur = [], [], [], 0

    for path in jsonl_paths:
        with open(path) as f:
            for line in f:
                if not line.strip():
                    continue
                ids, m = encode_chat(json.loads(line)[messages_key], tok)
                ids.append(tok.eos_id)
                m.append(0)
                toks.append(np.asarray(ids, dtype=np.uint32))
                masks.append(np.asarray(m, dtype=np.uint8))
                cur += len(ids)
                ends.append(cur)
                total += len(ids)
                n_docs += 1
                if cur >= shard_tokens:
                    flush()
    flush()
    meta = {"shards": shards, "num_tokens": total, "num_docs": n_docs, "format": "chat", "eos_id": tok.eos_id,
            "vocab_size": tok.vocab_size}
    with open(os.path.join(cache_path, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    with open(os.path.join(cache_path, ".success"), "w") as f:
        f.write("ok\n")
    return meta
