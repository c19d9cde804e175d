"""Train this project's own tokenizers: a domain-weighted raw-text corpus, plain BPE / SuperBPE
arms trained on it, exported as Hugging Face ``tokenizer.json`` + ``tokenizer_config.json`` and
published to a tokenizer mirror that ``data.tokenize.load_tokenizer("trained/<name>")`` reads
(tokenization/corpus.py:74-182, tokenization/train_tokenizer.py:66-362).

* ``build_corpus(source_root, out_dir)``: each domain of ``TRAIN_DOMAINS`` (English web, code,
  several languages, math) gets ``total_bytes`` x its weight, split evenly over its sources; from
  each source the first ``skip_bytes`` are skipped (they stay unseen, for a held-out fertility
  sample) and then documents are copied until the budget is met. A domain is one
  ``<domain>.jsonl.gz`` of ``{"text"}`` rows; ``manifest.json`` records what was written per source.
  A source that cannot be read is recorded with its error and skipped, not fatal. Sources are read
  from local snapshots (``<source_root>/<hf id>/<config>/``, or ``<hf id>/`` for a dataset without configs,
  with Parquet or JSON-lines files): the
  machines here have no network.
* ``TrainSpec(name, kind, vocab_size, transition_vocab)`` and ``train_one(spec, texts, out_dir)``:
  ``bpe`` is the stock byte-level BPE trainer at ``vocab_size``; ``superbpe`` trains stage 1 to
  ``transition_vocab`` on the whole corpus and learns superword merges up to ``vocab_size`` on a
  bounded, evenly strided sample of it (stage 2's cost grows with the text it counts pairs over).
  Returns the vocabulary sizes, the fertility on held-out text and the time taken.
* ``publish(out_dir, mirror_root, name)`` copies the two files to
  ``<mirror_root>/tokenizers/trained/<name>/``; ``MXK_TOKENIZER_MIRROR`` points the loader there.
"""

from __future__ import annotations

import glob
import gzip
import json
import math
import os
import shutil
import time
from dataclasses import dataclass

EOS_TOKEN = "<|endoftext|>"

# (dataset id, config, split, text field): the public sources of the reference's training corpus.
TRAIN_DOMAINS: dict[str, tuple[tuple[str, str | None, str, str], ...]] = {
    "english_web": (("DKYoon/SlimPajama-6B", None, "train", "text"),),
    "code": (("codeparrot/codeparrot-clean-valid", None, "train", "content"),),
    "multilingual": tuple(("wikimedia/wikipedia", f"20231101.{lang}", "train", "text")
                          for lang in ("de", "fr", "es", "ru", "zh", "ja", "ar", "hi")),
    "math": (("HuggingFaceTB/finemath", "finemath-3plus", "train", "text"),),
}
DOMAIN_WEIGHTS = {"english_web": 0.50, "code": 0.20, "multilingual": 0.20, "math": 0.10}
TOTAL_BYTES = 4_000_000_000
SKIP_BYTES = 20_000_000


def _source_files(root: str, hf_id: str, config: str | None, split: str) -> list[str]:
    base = os.path.join(root, hf_id, config or "")
    if not os.path.isdir(base):
        raise FileNotFoundError(f"no local snapshot of {hf_id} ({config}) under {base}")
    files = sorted(p for ext in ("parquet", "jsonl", "jsonl.gz")
                   for p in glob.glob(os.path.join(base, "**", f"*.{ext}"), recursive=True))
    return [p for p in files if split in os.path.relpath(p, base)] or files


def _iter_texts(files: list[str], field: str):
    from ..data.instruct import _read_file

    for f in files:
        for row in _read_file(f):
            t = row.get(field) or ""
            if t:
                yield t


def build_corpus(source_root: str, out_dir: str, total_bytes: int = TOTAL_BYTES,
                 weights: dict[str, float] | None = None, skip_bytes: int = SKIP_BYTES,
                 domains: dict | None = None) -> dict:
    weights = dict(weights or DOMAIN_WEIGHTS)
    domains = domains or TRAIN_DOMAINS
    os.makedirs(out_dir, exist_ok=True)
    manifest = {"total_bytes": total_bytes, "skip_bytes": skip_bytes, "domains": {}}
    for dom, w in weights.items():
        specs = domains[dom]
        budget = max(1, int(total_bytes * w) // len(specs))
        path = os.path.join(out_dir, f"{dom}.jsonl.gz")
        tmp = path + ".tmp"
        srcs, d_bytes, d_docs = [], 0, 0
        with gzip.open(tmp, "wt", encoding="utf-8") as out:
            for hf_id, config, split, field in specs:
                wrote = skipped = docs = 0
                try:
                    for text in _iter_texts(_source_files(source_root, hf_id, config, split), field):
                        n = len(text.encode("utf-8"))
                        if skipped < skip_bytes:
                            skipped += n
                            continue
                        out.write(json.dumps({"text": text}, ensure_ascii=False) + "\n")
                        wrote += n
                        docs += 1
                        if wrote >= budget:
                            break
                except Exception as e:  # a missing or unreadable source is recorded, not fatal
                    srcs.append({"source": hf_id, "config": config, "bytes": wrote, "docs": docs, "error": str(e)})
                else:
                    srcs.append({"source": hf_id, "config": config, "bytes": wrote, "docs": docs})
                d_bytes += wrote
                d_docs += docs
        os.replace(tmp, path)
        manifest["domains"][dom] = {"file": os.path.basename(path), "bytes": d_bytes, "docs": d_docs,
                                    "sources": srcs}
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return manifest


def read_corpus(corpus_dir: str, domains: tuple[str, ...] | None = None) -> list[str]:
    doms = domains or tuple(DOMAIN_WEIGHTS)
    texts = []
    for d in doms:
        p = os.path.join(corpus_dir, f"{d}.jsonl.gz")
        if os.path.exists(p):
            with gzip.open(p, "rt", encoding="utf-8") as f:
                texts += [json.loads(line)["text"] for line in f if line.strip()]
    return texts


@dataclass(frozen=True)
class TrainSpec:
    name: str
    kind: str = "bpe"  # bpe | superbpe
    vocab_size: int = 128_000
    transition_vocab: int = 0  # superbpe: the stage-1 size (0 -> 80 % of vocab_size)
    stage2_max_bytes: int = 60_000_000


def _bounded_sample(texts: list[str], max_bytes: int) -> list[str]:
    """Every k-th document, k chosen so the sample is about ``max_bytes`` (all of them when smaller)."""
    total = sum(len(t.encode("utf-8")) for t in texts)
    if total <= max_bytes:
        return texts
    return texts[::math.ceil(total / max_bytes)]


def save_tokenizer(tok, out_dir: str, model_max_length: int = 131072) -> None:
    os.makedirs(out_dir, exist_ok=True)
    tok.save(os.path.join(out_dir, "tokenizer.json"))
    cfg = {"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": EOS_TOKEN, "bos_token": None,
           "unk_token": None, "model_max_length": model_max_length, "clean_up_tokenization_spaces": False}
    with open(os.path.join(out_dir, "tokenizer_config.json"), "w") as f:
        json.dump(cfg, f, indent=1)


def train_one(spec: TrainSpec, texts: list[str], out_dir: str, held_out: list[str] | None = None) -> dict:
    from .superbpe import extend_with_superwords, fertility, train_plain_bpe

    t0 = time.time()
    if spec.kind == "bpe":
        tok = train_plain_bpe(texts, spec.vocab_size, special_tokens=(EOS_TOKEN,))
        stats = {"stage1_vocab": tok.get_vocab_size()}
    elif spec.kind == "superbpe":
        trans = spec.transition_vocab or int(0.8 * spec.vocab_size)
        if not 0 < trans < spec.vocab_size:
            raise ValueError(f"{spec.name}: transition_vocab {trans} must lie below vocab_size {spec.vocab_size}")
        stage1 = train_plain_bpe(texts, trans, special_tokens=(EOS_TOKEN,))
        res = extend_with_superwords(stage1, _bounded_sample(texts, spec.stage2_max_bytes), spec.vocab_size)
        tok = res.tokenizer
        stats = {"stage1_vocab": res.transition_vocab, "superword_merges": res.n_superword_merges}
    else:
        raise ValueError(f"unknown tokenizer kind {spec.kind!r}")
    save_tokenizer(tok, out_dir)
    out = {"name": spec.name, "kind": spec.kind, "vocab_size": tok.get_vocab_size(), "seconds": time.time() - t0,
           **stats}
    if held_out:
        out["fertility"] = fertility(tok, held_out)
    with open(os.path.join(out_dir, "train_stats.json"), "w") as f:
        json.dump(out, f, indent=1)
    return out


def publish(out_dir: str, mirror_root: str, name: str) -> str:
    dest = os.path.join(mirror_root, "tokenizers", "trained", name)
    os.makedirs(dest, exist_ok=True)
    for fn in ("tokenizer.json", "tokenizer_config.json"):
        shutil.copy(os.path.join(out_dir, fn), os.path.join(dest, fn))
    return dest


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(prog="python -m marin_experiments_b200.tokenization.train")
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("corpus", help="build the raw-text corpus from local snapshots")
    c.add_argument("--sources", required=True)
    c.add_argument("--out", required=True)
    c.add_argument("--total-bytes", type=float, default=TOTAL_BYTES)
    t = sub.add_parser("train", help="train one arm on a corpus and publish it")
    t.add_argument("--corpus", required=True)
    t.add_argument("--name", required=True)
    t.add_argument("--kind", choices=["bpe", "superbpe"], default="bpe")
    t.add_argument("--vocab", type=int, default=128_000)
    t.add_argument("--transition", type=int, default=0)
    t.add_argument("--out", required=True)
    t.add_argument("--mirror", default=os.environ.get("MXK_TOKENIZER_MIRROR", ""))
    a = ap.parse_args(argv)
    if a.cmd == "corpus":
        print(json.dumps(build_corpus(a.sources, a.out, int(a.total_bytes)), indent=1))
        return 0
    stats = train_one(TrainSpec(a.name, a.kind, a.vocab, a.transition), read_corpus(a.corpus), a.out)
    print(json.dumps(stats, indent=1))
    if a.mirror:
        print("published to", publish(a.out, a.mirror, a.name))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
