"""Speech tokens for ASR-style LM training (speech-asr/audio_tokens.py:33-139, speech-asr/bpe.py:50-167).

* ``flatten_codes``: neural-codec codes ``[codebooks, frames]`` flattened time-major (frame outer,
  codebook inner), the layout the reference writes.
* ``encode_with_codec``: runs a local Hugging Face Mimi checkpoint (``transformers.MimiModel``) over
  waveforms after a linear resample to the codec rate (there is no network: a local model directory
  is required).
* ``corpus_line``: ``"A_12 A_501 ... <sep> transcript"`` -- each code as a prefixed word, then the
  separator and the lower-cased transcript.
* ``train_audio_bpe``: a byte-level BPE over such lines (stock ``tokenizers``), with the pad / bos /
  eos / separator specials, so frequent code n-grams merge into single tokens.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence

import numpy as np


def flatten_codes(codes) -> list[int]:
    a = np.asarray(codes)
    if a.ndim != 2:
        raise ValueError("codes must be [codebooks, frames]")
    return a.transpose(1, 0).reshape(-1).astype(np.int64).tolist()


def unflatten_codes(flat: Sequence[int], num_codebooks: int) -> np.ndarray:
    a = np.asarray(flat, dtype=np.int64)
    if a.size % num_codebooks:
        raise ValueError("length is not a multiple of the codebook count")
    return a.reshape(-1, num_codebooks).transpose(1, 0)


def resample_linear(samples: np.ndarray, src_sr: int, dst_sr: int) -> np.ndarray:
    if src_sr == dst_sr:
        return samples
    dur = samples.shape[0] / src_sr
    n = int(round(dur * dst_sr))
    t_src = np.arange(samples.shape[0], dtype=np.float64) / src_sr
    t_dst = np.arange(n, dtype=np.float64) / dst_sr
    return np.interp(t_dst, t_src, samples).astype(samples.dtype)


def encode_with_codec(waves: list[np.ndarray], srs: list[int], model_dir: str, num_codebooks: int = 8,
                      device: str = "cpu") -> list[list[int]]:
    import torch
    from transformers import AutoFeatureExtractor, MimiModel

    fe = AutoFeatureExtractor.from_pretrained(model_dir, local_files_only=True)
    model = MimiModel.from_pretrained(model_dir, local_files_only=True).to(device).eval()
    target = fe.sampling_rate
    wav = [resample_linear(w.astype(np.float32), sr, target) for w, sr in zip(waves, srs)]
    inputs = fe(raw_audio=wav, sampling_rate=target, return_tensors="pt", padding=True)
    with torch.no_grad():
        enc = model.encode(inputs["input_values"].to(device), padding_mask=inputs.get("padding_mask"),
                           num_quantizers=num_codebooks)
    codes = enc.audio_codes.to(torch.int64).cpu().numpy()
    return [flatten_codes(c) for c in codes]


def corpus_line(tokens: Sequence[int], transcript: str | None, prefix: str = "A_", sep: str = "<sep>") -> str:
    audio = " ".join(f"{prefix}{t}" for t in tokens)
    return f"{audio} {sep} {(transcript or '').strip().lower()}"


def train_audio_bpe(lines: Iterable[str], vocab_size: int, min_frequency: int = 2,
                    specials=("<pad>", "<s>", "</s>", "<sep>")):
    from tokenizers import ByteLevelBPETokenizer

    tok = ByteLevelBPETokenizer()
    tok.train_from_iterator(list(lines), vocab_size=vocab_size, min_frequency=min_frequency,
                            special_tokens=list(specials), show_progress=False)
    return tok
