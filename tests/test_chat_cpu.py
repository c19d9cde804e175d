"""ChatML SFT encoding: assistant-only loss masks reach the native loader's loss weights; corpus
recipes resolve local caches."""

import json

import pytest
import torch

from marin_experiments_b200.data.chat import encode_chat, render_chatml, write_chat_cache
from marin_experiments_b200.data.loader import open_cache
from marin_experiments_b200.data.tokenize import ByteTokenizer


def test_mask_covers_assistant_only(tmp_path):
    tok = ByteTokenizer()
    msgs = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"}]
    ids, mask = encode_chat(msgs, tok)
    assert tok.decode(ids) == render_chatml(msgs)
    trained = tok.decode([i for i, m in zip(ids, mask) if m])
    assert trained == "yo<|im_end|>\n"
    src = tmp_path / "c.jsonl"
    src.write_text(json.dumps({"messages": msgs}) + "\n")
    meta = write_chat_cache([str(src)], str(tmp_path / "cache"), tok)
    n = meta["num_tokens"]
    ds = open_cache(str(tmp_path / "cache"), n - 1, seed=0, shuffle=False)
    t = torch.empty(1, n - 1, dtype=torch.int32)
    g = torch.empty_like(t)
    w = torch.empty(1, n - 1)
    ds.fill_batch(0, t, g, w, 1)
    # weight at p trains the prediction of token p + 1: exactly the masked tokens
    want = torch.tensor(mask[1:n - 1] + [0], dtype=torch.float32)[: n - 1]
    want[-1] = 0
    assert torch.equal(w[0], want)


def test_recipe(tmp_path):
    from marin_experiments_b200.data.corpora import Recipe

    (tmp_path / "a").mkdir()
    (tmp_path / "a" / "meta.json").write_text("{}")
    r = Recipe("x", {"a": ("a", 0.5), "b": ("b", 0.5)})
    cfg = r.data_config(str(tmp_path))
    assert [c[0] for c in cfg.components] == ["a"]
    with pytest.raises(FileNotFoundError):
        r.data_config(str(tmp_path), missing="error")
