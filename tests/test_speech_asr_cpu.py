"""The speech pipeline end to end on CPU: tone clips -> random-init Mimi codes -> BPE -> token cache
-> two training steps of the ~30M grug."""

import json
import math
import os

import numpy as np
import pyarrow.parquet as pq
import pytest

from marin_experiments_b200.executor import Executor
from marin_experiments_b200.experiments import speech_asr


def test_wav_roundtrip(tmp_path):
    x = (0.5 * np.sin(np.linspace(0, 50, 4000))).astype(np.float32)
    speech_asr.write_wav(str(tmp_path / "a.wav"), x, 16000)
    y, sr = speech_asr.read_wav(str(tmp_path / "a.wav"))
    assert sr == 16000 and np.abs(y - x).max() < 1e-4


@pytest.mark.timeout(600)
def test_speech_pipeline(tmp_path, capsys, monkeypatch):
    monkeypatch.delenv("MIMI_MODEL_DIR", raising=False)
    monkeypatch.delenv("SPEECH_AUDIO_DIR", raising=False)
    monkeypatch.setenv("SPEECH_BPE_VOCAB", "400")
    steps = speech_asr.build_steps(steps=2, batch_size=2)
    res = Executor(str(tmp_path)).run(steps)
    t = pq.read_table(os.path.join(res["audio-tokens/speech-mimi"], "mimi-00000-of-00001.parquet")).to_pydict()
    assert len(t["id"]) == 20 and all(len(c) % 8 == 0 and len(c) > 0 for c in t["mimi_tokens"])
    assert len({c for row in t["mimi_tokens"] for c in row}) > 1  # random codebooks give varied codes
    assert all(s and s.isupper() for s in t["text"])
    meta = json.load(open(os.path.join(res["tokenized/speech"], "meta.json")))
    assert meta["vocab_size"] <= 400 and meta["num_docs"] == 20
    toks = np.fromfile(os.path.join(res["tokenized/speech"], meta["shards"][0]["tokens"]), dtype="<u4")
    from marin_experiments_b200.data.tokenize import load_tokenizer

    tok = load_tokenizer(res["bpe/speech-mimi"])
    assert toks[0] == tok.bos_id and tok.eos_id in toks
    out = capsys.readouterr().out
    assert out.count("[THRUPUT] step=") == 2
    train_dir = res["speech-asr/speech-30m"]
    metrics = [json.loads(l) for l in open(os.path.join(train_dir, "logs", "speech-asr-30m-cpu", "metrics.jsonl"))]
    assert [m["step"] for m in metrics] == [1, 2] and all(math.isfinite(m["train/loss"]) for m in metrics)
