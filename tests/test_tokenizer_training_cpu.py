"""Tokenizer training track: the domain-weighted corpus from local snapshots, BPE and SuperBPE arms,
export and the trained-tokenizer mirror."""

import gzip
import json
import os

import pytest

from marin_experiments_b200.tokenization import train as TT


def _snap(root, hf_id, config, split, field, texts, kind="jsonl"):
    d = os.path.join(root, hf_id, config or "", split)
    os.makedirs(d, exist_ok=True)
    if kind == "parquet":
        import pyarrow as pa
        import pyarrow.parquet as pq

        pq.write_table(pa.Table.from_pylist([{field: t} for t in texts]), os.path.join(d, "part-0.parquet"))
    else:
        with open(os.path.join(d, "part-0.jsonl"), "w") as f:
            for t in texts:
                f.write(json.dumps({field: t}) + "\n")


WORDS = "the of and a to in is was for on that with as by at from his her it an were are which".split()


def _docs(rng, n, lang=""):
    return [" ".join(rng.choice(WORDS) for _ in range(rng.randint(20, 60))) + f" {lang}{i}." for i in range(n)]


def test_corpus_budget_skip_and_errors(tmp_path):
    import random

    rng = random.Random(0)
    src = str(tmp_path / "src")
    doms = {"english_web": (("web/a", None, "train", "text"),),
            "code": (("code/b", None, "train", "content"),),
            "multilingual": (("wiki", "de", "train", "text"), ("wiki", "fr", "train", "text"),
                             ("wiki", "xx", "train", "text"))}  # the last one has no snapshot
    _snap(src, "web/a", None, "train", "text", _docs(rng, 400), "parquet")
    _snap(src, "web/a", None, "validation", "text", ["held out " * 20] * 5)
    _snap(src, "code/b", None, "train", "content", ["def f(x):\n    return x + 1\n" * 5] * 300)
    _snap(src, "wiki", "de", "train", "text", _docs(rng, 200, "de"))
    _snap(src, "wiki", "fr", "train", "text", _docs(rng, 200, "fr"))
    out = str(tmp_path / "corpus")
    man = TT.build_corpus(src, out, total_bytes=60_000, weights={"english_web": 0.5, "code": 0.2, "multilingual": 0.3},
                          skip_bytes=2_000, domains=doms)
    web = man["domains"]["english_web"]
    assert 30_000 <= web["bytes"] < 31_000 and web["sources"][0]["docs"] > 0
    ml = man["domains"]["multilingual"]["sources"]
    assert [s["config"] for s in ml] == ["de", "fr", "xx"] and "error" in ml[2] and ml[0]["bytes"] >= 6_000
    texts = TT.read_corpus(out, ("english_web", "code", "multilingual"))
    assert not any("held out" in t for t in texts)  # other splits are not read
    first_web = [json.loads(x)["text"] for x in gzip.open(os.path.join(out, "english_web.jsonl.gz"), "rt")][0]
    assert first_web != _docs(__import__("random").Random(0), 1)[0]  # the skipped prefix is not copied
    assert json.load(open(os.path.join(out, "manifest.json"))) == man


def test_train_arms_publish_and_load(tmp_path, monkeypatch):
    import random

    rng = random.Random(1)
    texts = _docs(rng, 300)
    held = _docs(rng, 20)
    bpe = TT.train_one(TT.TrainSpec("t-bpe", "bpe", 400), texts, str(tmp_path / "bpe"), held)
    sup = TT.train_one(TT.TrainSpec("t-super", "superbpe", 500, 400), texts, str(tmp_path / "super"), held)
    assert bpe["vocab_size"] <= 401 and sup["stage1_vocab"] <= 401 and sup["superword_merges"] > 0  # + the end token
    assert sup["fertility"]["bytes_per_token"] > bpe["fertility"]["bytes_per_token"]  # superwords span words
    cfg = json.load(open(tmp_path / "super" / "tokenizer_config.json"))
    assert cfg["eos_token"] == TT.EOS_TOKEN
    with pytest.raises(ValueError, match="transition_vocab"):
        TT.train_one(TT.TrainSpec("bad", "superbpe", 300, 400), texts, str(tmp_path / "bad"))
    dest = TT.publish(str(tmp_path / "super"), str(tmp_path / "mirror"), "t-super")
    assert os.path.exists(os.path.join(dest, "tokenizer.json"))
    from marin_experiments_b200.data.tokenize import load_tokenizer

    monkeypatch.delenv("MXK_TOKENIZER_MIRROR", raising=False)
    with pytest.raises(FileNotFoundError, match="MXK_TOKENIZER_MIRROR"):
        load_tokenizer("trained/t-super")
    monkeypatch.setenv("MXK_TOKENIZER_MIRROR", str(tmp_path / "mirror"))
    tok = load_tokenizer("trained/t-super")
    s = "the of and a to in"
    assert tok.decode(tok.encode(s)) == s and tok.eos_id == tok.tok.token_to_id(TT.EOS_TOKEN)
