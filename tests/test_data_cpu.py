"""Native data pipeline: permutation, synthetic examples, token cache windows and packing,
block mixtures, and the prefetching loader."""

import json
import os

import numpy as np
import pytest
import torch

from marin_experiments_b200.config import DataConfig
from marin_experiments_b200.data.loader import DataLoader, build_dataset, mixture_weights_at, open_cache
from marin_experiments_b200.data.tokenize import ByteTokenizer, TokenizeConfig, tokenize
from marin_experiments_b200.runtime import rt


def _batch(ds, first, n):
    s = ds.seq_len()
    t = torch.empty(n, s, dtype=torch.int32)
    g = torch.empty(n, s, dtype=torch.int32)
    w = torch.empty(n, s, dtype=torch.float32)
    ds.fill_batch(first, t, g, w, 2)
    return t, g, w


@pytest.mark.parametrize("n", [1, 2, 7, 100, 1000, 4097])
def test_permutation_is_bijection(n):
    out = sorted(rt().permutation(n, 1234, i) for i in range(n))
    assert out == list(range(n))


def test_synthetic_deterministic_and_packed():
    ds = rt().SyntheticDataset(64, 1000, 16, 3)
    t1, g1, w1 = _batch(ds, 10, 4)
    t2, _, _ = _batch(ds, 10, 4)
    assert torch.equal(t1, t2)
    assert t1.min() >= 1 and t1.max() < 1000
    assert torch.equal(g1[0], torch.arange(64, dtype=torch.int32) // 16)
    # no loss across document boundaries or at the last position
    assert w1[0, 15] == 0 and w1[0, 14] == 1 and w1[0, 63] == 0
    t3, _, _ = _batch(ds, 11, 1)
    assert not torch.equal(t1[1:2], t1[0:1]) and torch.equal(t3[0], t1[1])


def _write_cache(tmp_path, docs):
    d = tmp_path / "cache"
    d.mkdir()
    toks = np.concatenate([np.asarray(x, dtype="<u4") for x in docs])
    ends = np.cumsum([len(x) for x in docs]).astype("<u8")
    toks.tofile(d / "tokens-00000.bin")
    ends.tofile(d / "docs-00000.bin")
    (d / "meta.json").write_text(json.dumps({"shards": [{"tokens": "tokens-00000.bin", "docs": "docs-00000.bin"}]}))
    return str(d)


def test_token_cache_windows_segments(tmp_path):
    docs = [list(range(100, 105)), list(range(200, 203)), list(range(300, 308))]  # 16 tokens
    path = _write_cache(tmp_path, docs)
    ds = open_cache(path, 8, seed=0, shuffle=False)
    assert ds.size() == 2
    t, g, w = _batch(ds, 0, 2)
    assert t[0].tolist() == [100, 101, 102, 103, 104, 200, 201, 202]
    assert g[0].tolist() == [0, 0, 0, 0, 0, 1, 1, 1]
    assert w[0].tolist() == [1, 1, 1, 1, 0, 1, 1, 0]
    assert t[1].tolist() == list(range(300, 308))
    # epochs wrap
    t2, _, _ = _batch(ds, 2, 1)
    assert torch.equal(t2[0], t[0])
    sh = open_cache(path, 8, seed=5, shuffle=True)
    ts, _, _ = _batch(sh, 0, 2)
    assert sorted(map(tuple, ts.tolist())) == sorted(map(tuple, t.tolist()))


def test_mixture_block_counts(tmp_path):
    m = rt()
    a = m.SyntheticDataset(8, 50, 8, 1)
    b = m.SyntheticDataset(8, 50, 8, 2)
    mix = m.MixtureDataset([a, b], [0, 64], [[0.75, 0.25], [0.0, 1.0]], 32, 7, 0)
    comps = [mix.resolve(i)[0] for i in range(64)]
    assert comps[:32].count(0) == 24 and comps[32:64].count(0) == 24
    assert all(mix.resolve(i)[0] == 1 for i in range(64, 128))
    # component-local indices are dense and increasing per component
    locals0 = sorted(mix.resolve(i)[1] for i in range(64) if mix.resolve(i)[0] == 0)
    assert locals0 == list(range(48))
    locals1 = sorted(mix.resolve(i)[1] for i in range(128) if mix.resolve(i)[0] == 1)
    assert locals1 == list(range(16 + 64))
    assert mixture_weights_at([(0, {"a": 1.0}), (10, {"a": 0.5})], 12) == {"a": 0.5}


def test_first_exhausted_stops(tmp_path):
    path = _write_cache(tmp_path, [list(range(1, 17))])
    cfg = DataConfig(source="cache", cache_dir=path, seed=0)
    ds = build_dataset(cfg, 8, 100, block_size=2, stop_strategy="first_exhausted")
    it = DataLoader(ds, 2, pin=False)
    next(it)
    with pytest.raises(StopIteration):
        next(it)


def test_loader_matches_direct_fill_and_ranks():
    cfg = DataConfig(source="synthetic", seed=4, doc_len=32)
    ds = build_dataset(cfg, 64, 5000, block_size=16)
    full = DataLoader(ds, 8, pin=False)
    r1 = DataLoader(ds, 8, rank=1, world=2, pin=False)
    for _ in range(3):
        b = next(full)
        tok = b["tokens"].clone()
        part = next(r1)
        assert torch.equal(part["tokens"], tok[4:])
    resumed = DataLoader(ds, 8, start_step=2, pin=False)
    assert torch.equal(next(resumed)["tokens"], tok)


def test_tokenize_step(tmp_path):
    src = tmp_path / "docs.jsonl"
    src.write_text("\n".join(json.dumps({"text": t}) for t in ["hello", "world!", "abc"]) + "\n")
    out = tmp_path / "tok"
    meta = tokenize(TokenizeConfig(train_paths=(str(src),), cache_path=str(out), sample_count=2))
    assert meta["num_docs"] == 2 and meta["num_tokens"] == len("hello") + len("world!") + 2
    assert os.path.exists(out / ".success")
    ds = open_cache(str(out), 4, seed=0, shuffle=False)
    t, g, _ = _batch(ds, 0, 1)
    assert ByteTokenizer().decode(t[0].tolist()) == "hell"
    again = tokenize(TokenizeConfig(train_paths=(str(src),), cache_path=str(out)))
    assert again["num_docs"] == 2  # complete cache: the step is skipped


def test_crc32c_known_value():
    # CRC-32C check value of "123456789" (RFC 3720 appendix)
    t = torch.tensor(list(b"123456789"), dtype=torch.uint8)
    assert rt().crc32c(t) == 0xE3069283
