import numpy as np

from marin_experiments_b200.data.audio_tokens import (corpus_line, flatten_codes, resample_linear, train_audio_bpe,
                                                      unflatten_codes)


def test_time_major_roundtrip_and_corpus():
    codes = np.arange(24).reshape(8, 3)  # 8 codebooks, 3 frames
    flat = flatten_codes(codes)
    assert flat[:8] == [0, 3, 6, 9, 12, 15, 18, 21]  # frame 0 across codebooks
    assert np.array_equal(unflatten_codes(flat, 8), codes)
    line = corpus_line([5, 7], "Hello World")
    assert line == "A_5 A_7 <sep> hello world"
    x = np.sin(np.linspace(0, 10, 1600)).astype(np.float32)
    assert resample_linear(x, 16000, 24000).shape[0] == 2400


def test_audio_bpe_merges_frequent_codes():
    rng = np.random.default_rng(0)
    lines = [corpus_line(rng.integers(0, 20, 40).tolist(), "the cat") for _ in range(200)]
    tok = train_audio_bpe(lines, vocab_size=400)
    enc = tok.encode(lines[0])
    assert len(enc.ids) < len(lines[0].split()) * 3
    assert tok.token_to_id("<sep>") is not None
