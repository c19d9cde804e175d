"""Speech-recognition language-model pipeline: audio -> neural-codec tokens -> BPE tokenizer ->
token cache -> ~30M dense grug (speech-asr/launch.py:1-330, speech-asr/audio_tokens.py:33-139,
speech-asr/bpe.py:50-167).

Steps (each an ``ExecutorStep`` with its own output directory, so reruns skip finished work):

1. ``audio``: 16-bit PCM WAV clips with transcripts. ``SPEECH_AUDIO_DIR`` names a directory of
   ``<id>.wav`` + ``<id>.txt`` pairs; without one (there is no network for LibriSpeech) a small
   deterministic corpus of tone sequences is written whose transcripts name the tones.
2. ``codec``: the neural audio codec. ``MIMI_MODEL_DIR`` names a local Hugging Face Mimi checkpoint
   (``kyutai/mimi``); without one a small randomly initialised Mimi (random codebooks, 8 quantizers)
   is saved instead: the pipeline then runs end to end, but its codes carry no phonetic meaning.
3. ``audio_tokens``: every clip resampled to the codec's rate and encoded to ``num_codebooks``
   code streams, flattened time-major (frame outer, codebook inner), written as parquet rows
   ``{id, mimi_tokens, text}`` like the reference's shards.
4. ``bpe``: corpus lines ``"A_c0 A_c1 ... <|sep|> transcript"`` and a byte-level BPE over them with
   the pad / bos / eos / separator specials; saved as ``tokenizer.json`` (plus the Hugging Face
   tokenizer files) and checked by a round trip.
5. ``tokenized``: the corpus through the tokenize step (begin- and end-of-sequence tokens added).
6. ``train``: the ~30M grug (hidden 128, 4 layers, 2 heads, ReLU MLP 448) with the vocabulary
   rounded up to a multiple of 128 and 4,096-token sequences (audio dominates: ~1,000 codec
   tokens per 10 s clip), AdamW 6e-4 cosine.

Run: ``python -m marin_experiments_b200.experiments.speech_asr --prefix /tmp/out [--dry_run]``.
"""

from __future__ import annotations

import glob
import json
import math
import os
import wave
from dataclasses import dataclass, replace

import numpy as np
import torch

from ..config import DataConfig, GrugTrainerConfig
from ..data.audio_tokens import corpus_line, encode_with_codec
from ..data.tokenize import TokenizeConfig, tokenize
from ..executor import ExecutorStep, executor_main, output_path_of, this_output_path, versioned
from ..optim import AdamConfig
from .common import GrugLaunchConfig, run_inline
from .tiny_stories import TINY_MODEL

SEP, PAD, BOS, EOS = "<|sep|>", "<|pad|>", "<|bos|>", "<|eos|>"


def _accelerator() -> str:
    return "gpu" if torch.cuda.is_available() else "cpu"


def bpe_vocab() -> int:
    return int(os.environ.get("SPEECH_BPE_VOCAB", "2048" if _accelerator() == "cpu" else "16384"))


def model_vocab(n: int) -> int:
    return ((n + 127) // 128) * 128


# ---------------------------------------------------------------------------------------- audio
def write_wav(path: str, samples: np.ndarray, sr: int) -> None:
    pcm = np.clip(samples, -1.0, 1.0)
    with wave.open(path, "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(sr)
        w.writeframes((pcm * 32767.0).astype("<i2").tobytes())


def read_wav(path: str) -> tuple[np.ndarray, int]:
    """Mono float32 samples in [-1, 1] and the rate of a 16-bit PCM WAV (channels averaged)."""
    with wave.open(path, "rb") as w:
        if w.getsampwidth() != 2:
            raise ValueError(f"{path}: only 16-bit PCM WAV is supported")
        sr, ch = w.getframerate(), w.getnchannels()
        a = np.frombuffer(w.readframes(w.getnframes()), dtype="<i2").astype(np.float32) / 32768.0
    return (a.reshape(-1, ch).mean(axis=1) if ch > 1 else a), sr


_TONES = {"low": 220.0, "mid": 440.0, "high": 880.0, "buzz": 150.0}


@dataclass(frozen=True)
class AudioConfig:
    output_path: str
    source: str | None = None
    num_clips: int = 20
    sample_rate: int = 16000
    seed: int = 0


def write_audio(cfg: AudioConfig) -> None:
    os.makedirs(cfg.output_path, exist_ok=True)
    if cfg.source:
        import shutil

        for f in sorted(glob.glob(os.path.join(cfg.source, "*.wav"))):
            shutil.copy(f, cfg.output_path)
            txt = f[:-4] + ".txt"
            if os.path.exists(txt):
                shutil.copy(txt, cfg.output_path)
        return
    rng = np.random.default_rng(cfg.seed)
    names = sorted(_TONES)
    for i in range(cfg.num_clips):
        words = [names[k] for k in rng.integers(0, len(names), rng.integers(2, 6))]
        seg = int(0.25 * cfg.sample_rate)
        t = np.arange(seg) / cfg.sample_rate
        parts = [0.4 * np.sin(2 * math.pi * _TONES[w] * t) * np.hanning(seg) for w in words]
        clip = np.concatenate(parts) + 0.01 * rng.standard_normal(seg * len(words))
        write_wav(os.path.join(cfg.output_path, f"clip{i:04d}.wav"), clip.astype(np.float32), cfg.sample_rate)
        with open(os.path.join(cfg.output_path, f"clip{i:04d}.txt"), "w") as f:
            f.write(" ".join(words).upper() + "\n")


# ---------------------------------------------------------------------------------------- codec
@dataclass(frozen=True)
class CodecConfig:
    output_path: str
    model_dir: str | None = None
    seed: int = 0


def prepare_codec(cfg: CodecConfig) -> None:
    """Record the codec to use: a local Mimi checkpoint, or a small random-init stand-in."""
    os.makedirs(cfg.output_path, exist_ok=True)
    if cfg.model_dir:
        with open(os.path.join(cfg.output_path, "codec.json"), "w") as f:
            json.dump({"model_dir": cfg.model_dir, "random_init": False}, f)
        return
    from transformers import EncodecFeatureExtractor, MimiConfig, MimiModel

    torch.manual_seed(cfg.seed)
    mc = MimiConfig(hidden_size=64, num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=4, head_dim=16,
                    intermediate_size=128, num_filters=8, codebook_size=256, codebook_dim=64,
                    vector_quantization_hidden_dimension=64, num_quantizers=8, num_semantic_quantizers=1,
                    sliding_window=32, upsample_groups=64)
    model = MimiModel(mc)
    for mod in model.modules():  # codebooks are running means: give them random centroids
        if hasattr(mod, "embed_sum") and hasattr(mod, "cluster_usage"):
            mod.embed_sum.normal_()
            mod.cluster_usage.fill_(1.0)
    d = os.path.join(cfg.output_path, "model")
    model.save_pretrained(d)
    EncodecFeatureExtractor(feature_size=1, sampling_rate=mc.sampling_rate, padding_value=0.0).save_pretrained(d)
    with open(os.path.join(cfg.output_path, "codec.json"), "w") as f:
        json.dump({"model_dir": d, "random_init": True}, f)


def codec_dir(codec_path: str) -> str:
    with open(os.path.join(codec_path, "codec.json")) as f:
        return json.load(f)["model_dir"]


@dataclass(frozen=True)
class AudioTokensConfig:
    input_path: str
    codec_path: str
    output_path: str
    num_codebooks: int = 8
    batch_size: int = 8
    max_samples: int | None = None


def encode_audio(cfg: AudioTokensConfig) -> None:
    import pyarrow as pa
    import pyarrow.parquet as pq

    os.makedirs(cfg.output_path, exist_ok=True)
    wavs = sorted(glob.glob(os.path.join(cfg.input_path, "*.wav")))
    if cfg.max_samples is not None:
        wavs = wavs[: cfg.max_samples]
    model_dir = codec_dir(cfg.codec_path)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    rows = {"id": [], "mimi_tokens": [], "text": []}
    for i in range(0, len(wavs), cfg.batch_size):
        batch = wavs[i: i + cfg.batch_size]
        audio = [read_wav(p) for p in batch]
        codes = encode_with_codec([a for a, _ in audio], [sr for _, sr in audio], model_dir, cfg.num_codebooks,
                                  device=dev)
        for p, c in zip(batch, codes):
            txt = p[:-4] + ".txt"
            rows["id"].append(os.path.basename(p)[:-4])
            rows["mimi_tokens"].append(c)
            rows["text"].append(open(txt).read().strip() if os.path.exists(txt) else "")
    pq.write_table(pa.table(rows), os.path.join(cfg.output_path, "mimi-00000-of-00001.parquet"))


# ---------------------------------------------------------------------------------------- BPE
@dataclass(frozen=True)
class BpeConfig:
    input_path: str
    output_path: str
    vocab_size: int = 2048
    min_frequency: int = 2
    audio_token_prefix: str = "A_"


def train_bpe(cfg: BpeConfig) -> None:
    import pyarrow.parquet as pq
    from tokenizers import ByteLevelBPETokenizer

    os.makedirs(cfg.output_path, exist_ok=True)
    lines = []
    for shard in sorted(glob.glob(os.path.join(cfg.input_path, "mimi-*.parquet"))):
        t = pq.read_table(shard).to_pydict()
        lines += [corpus_line(toks, text, cfg.audio_token_prefix, SEP) for toks, text in zip(t["mimi_tokens"], t["text"])]
    if not lines:
        raise RuntimeError(f"no codec-token shards under {cfg.input_path}")
    with open(os.path.join(cfg.output_path, "corpus-00000.jsonl"), "w") as f:
        for ln in lines:
            f.write(json.dumps({"text": ln}) + "\n")
    tok = ByteLevelBPETokenizer()
    tok.train_from_iterator(lines, vocab_size=cfg.vocab_size, min_frequency=cfg.min_frequency,
                            special_tokens=[PAD, BOS, EOS, SEP], show_progress=False)
    tok.save(os.path.join(cfg.output_path, "tokenizer.json"))
    from transformers import PreTrainedTokenizerFast

    hf = PreTrainedTokenizerFast(tokenizer_file=os.path.join(cfg.output_path, "tokenizer.json"), pad_token=PAD,
                                 bos_token=BOS, eos_token=EOS, sep_token=SEP)
    hf.save_pretrained(cfg.output_path)
    sample = f"{cfg.audio_token_prefix}1 {cfg.audio_token_prefix}2 {SEP} hello world"
    ids = hf.encode(sample, add_special_tokens=False)
    if not ids or not hf.decode(ids).strip():
        raise RuntimeError("saved tokenizer does not round-trip a sample line")


# ---------------------------------------------------------------------------------------- steps
def build_steps(steps: int | None = None, batch_size: int | None = None) -> list[ExecutorStep]:
    cpu = _accelerator() == "cpu"
    audio = ExecutorStep(name="raw/speech-audio", fn=write_audio,
                         config=AudioConfig(output_path=this_output_path(),
                                            source=os.environ.get("SPEECH_AUDIO_DIR") or None))
    codec = ExecutorStep(name="codec/mimi", fn=prepare_codec,
                         config=CodecConfig(output_path=this_output_path(),
                                            model_dir=os.environ.get("MIMI_MODEL_DIR") or None))
    tokens = ExecutorStep(name="audio-tokens/speech-mimi", fn=encode_audio,
                          config=AudioTokensConfig(input_path=output_path_of(audio), codec_path=output_path_of(codec),
                                                   output_path=this_output_path(), num_codebooks=versioned(8),
                                                   batch_size=versioned(2 if cpu else 8),
                                                   max_samples=versioned(20 if cpu else None)))
    vocab = bpe_vocab()
    bpe = ExecutorStep(name="bpe/speech-mimi", fn=train_bpe,
                       config=BpeConfig(input_path=output_path_of(tokens), output_path=this_output_path(),
                                        vocab_size=versioned(vocab), min_frequency=versioned(2)))
    tokenized = ExecutorStep(name="tokenized/speech", fn=tokenize,
                             config=TokenizeConfig(train_paths=(output_path_of(bpe),), cache_path=this_output_path(),
                                                   tokenizer=output_path_of(bpe), prepend_bos=True,
                                                   sample_count=versioned(1_000 if cpu else None)))
    seq = 256 if cpu else 4096
    model = replace(TINY_MODEL, vocab_size=model_vocab(vocab), max_seq_len=seq, sliding_window=seq)
    launch = GrugLaunchConfig(
        model=versioned(model),
        data=DataConfig(source="cache", cache_dir=output_path_of(tokenized), seed=0),
        output_path=this_output_path(), run_id=os.environ.get("GRUG_RUN_ID", f"speech-asr-30m-{_accelerator()}"),
        steps=versioned(steps or int(os.environ.get("SPEECH_ASR_STEPS", "1" if cpu else "2000"))),
        batch_size=versioned(batch_size or (8 if cpu else 128)),
        seed=versioned(0),
        mp=versioned("params=float32,compute=float32,output=float32" if cpu
                     else "params=float32,compute=bfloat16,output=bfloat16"),
        optimizer=versioned(AdamConfig(learning_rate=6e-4, weight_decay=0.1, lr_schedule="cosine", decay=0.2,
                                       min_lr_ratio=0.1, warmup=0.1 if cpu else 200)),
        grug_trainer=versioned(GrugTrainerConfig(z_loss_weight=1e-4, ema_beta=None, log_every=1)),
        save_interval_s=600, keep=({"every": 1000},), eval=None,
    )
    train = ExecutorStep(name="speech-asr/speech-30m", fn=run_inline, config=launch)
    return [audio, codec, tokens, bpe, tokenized, train]


def main(argv=None):
    return executor_main(build_steps(), description=f"speech-asr: codec tokens -> BPE -> ~30M grug ({_accelerator()})",
                         argv=argv)


if __name__ == "__main__":
    main()
