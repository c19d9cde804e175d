"""Plain BPE and SuperBPE tokenizer training (tokenization/superbpe.py:1-365; SuperBPE: Liu et al.,
arXiv:2503.13423).

Stage 1 trains an ordinary byte-level BPE with the stock ``tokenizers`` trainer; its pre-tokenizer
keeps words apart (the GPT-2 byte-level rule), so no merge spans a word boundary. Stage 2 continues
merging past the transition vocabulary size on a permissive segmentation -- runs of text split only
at newlines, digit runs and punctuation runs -- so merges can join several words ("superwords" such
as `` of the``). Each stage-2 segment is first encoded with the stage-1 model; a greedy pair-merge
learner over those stage-1 token ids (counting pairs weighted by segment frequency and updating the
counts incrementally as it merges) adds merges until the final vocabulary size. The result is one
BPE tokenizer whose merge list is the stage-1 merges followed by the superword merges, with the
permissive pre-tokenizer; applying merges by rank reproduces both stages.
"""

from __future__ import annotations

import json
from collections import Counter, defaultdict
from collections.abc import Iterable
from dataclasses import dataclass

from tokenizers import Regex, Tokenizer, decoders, pre_tokenizers
from tokenizers.models import BPE
from tokenizers.trainers import BpeTrainer

# stage 2: keep text together, isolating digit runs, punctuation runs and newlines
STAGE2_REGEX = r"\p{N}+|[^\s\p{L}\p{N}]+|\r?\n| ?[^\r\n\p{N}\p{P}\p{S}]+"


def _byte_level(use_regex: bool = True):
    return pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=use_regex)


def train_plain_bpe(texts: Iterable[str], vocab_size: int, special_tokens=("<|endoftext|>",)) -> Tokenizer:
    tok = Tokenizer(BPE())
    tok.pre_tokenizer = _byte_level()
    tok.decoder = decoders.ByteLevel()
    trainer = BpeTrainer(vocab_size=vocab_size, special_tokens=list(special_tokens),
                         initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(list(texts), trainer=trainer)
    return tok


def _stage2_segments(texts: Iterable[str]) -> Counter:
    split = pre_tokenizers.Split(Regex(STAGE2_REGEX), behavior="isolated")
    seg = Counter()
    for t in texts:
        for piece, _ in split.pre_tokenize_str(t):
            if piece:
                seg[piece] += 1
    return seg


def _learn_merges(seqs: list[list[int]], freqs: list[int], n_merges: int, next_id: int):
    """Greedy BPE over token-id sequences: returns [(a, b, new_id)] in merge order."""
    pair_count: dict[tuple[int, int], int] = defaultdict(int)
    where: dict[tuple[int, int], set[int]] = defaultdict(set)
    for i, (s, f) in enumerate(zip(seqs, freqs)):
        for a, b in zip(s, s[1:]):
            pair_count[(a, b)] += f
            where[(a, b)].add(i)
    merges = []
    for _ in range(n_merges):
        if not pair_count:
            break
        best = max(pair_count.items(), key=lambda kv: (kv[1], -kv[0][0], -kv[0][1]))
        (a, b), cnt = best
        if cnt < 2:
            break
        new = next_id
        next_id += 1
        merges.append((a, b, new))
        for i in list(where.pop((a, b), ())):
            s, f = seqs[i], freqs[i]
            for x, y in zip(s, s[1:]):  # remove this sequence's old pairs
                pair_count[(x, y)] -= f
                if pair_count[(x, y)] <= 0:
                    pair_count.pop((x, y), None)
                where[(x, y)].discard(i)
            out, j = [], 0
            while j < len(s):
                if j + 1 < len(s) and s[j] == a and s[j + 1] == b:
                    out.append(new)
                    j += 2
                else:
                    out.append(s[j])
                    j += 1
            seqs[i] = out
            for x, y in zip(out, out[1:]):
                pair_count[(x, y)] += f
                where[(x, y)].add(i)
        pair_count.pop((a, b), None)
    return merges


@dataclass
class SuperBpeResult:
    tokenizer: Tokenizer
    transition_vocab: int
    final_vocab: int
    n_superword_merges: int


def extend_with_superwords(stage1: Tokenizer, texts: Iterable[str], final_vocab: int) -> SuperBpeResult:
    texts = list(texts)
    state = json.loads(stage1.to_str())
    vocab: dict[str, int] = state["model"]["vocab"]
    merges = state["model"]["merges"]
    id2tok = {i: t for t, i in vocab.items()}
    seg = _stage2_segments(texts)
    pieces = list(seg)
    seqs = [stage1.encode(p, add_special_tokens=False).ids for p in pieces]
    freqs = [seg[p] for p in pieces]
    n0 = len(vocab) + len(stage1.get_added_tokens_decoder())
    learned = _learn_merges(seqs, freqs, max(0, final_vocab - n0), max(id2tok) + 1)
    for a, b, new in learned:
        ta, tb = id2tok[a], id2tok[b]
        vocab[ta + tb] = new
        id2tok[new] = ta + tb
        merges.append([ta, tb] if isinstance(merges[0], list) else f"{ta} {tb}")
    state["model"]["vocab"] = vocab
    state["model"]["merges"] = merges
    state["pre_tokenizer"] = {"type": "Sequence", "pretokenizers": [
        {"type": "Split", "pattern": {"Regex": STAGE2_REGEX}, "behavior": "Isolated", "invert": False},
        {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": False}]}
    tok = Tokenizer.from_str(json.dumps(state))
    return SuperBpeResult(tok, n0, tok.get_vocab_size(), len(learned))


def fertility(tok: Tokenizer, texts: Iterable[str]) -> dict:
    """Tokens per byte and bytes per token of ``texts``."""
    n_tok = n_bytes = 0
    for t in texts:
        n_tok += len(tok.encode(t, add_special_tokens=False).ids)
        n_bytes += len(t.encode("utf-8"))
    return {"tokens_per_byte": n_tok / max(n_bytes, 1), "bytes_per_token": n_bytes / max(n_tok, 1),
            "tokens": n_tok, "bytes": n_bytes}
