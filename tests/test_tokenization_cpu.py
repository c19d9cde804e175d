"""Plain BPE and SuperBPE training: superword merges appear, fertility drops, round trips hold."""

import random

from marin_experiments_b200.tokenization.superbpe import extend_with_superwords, fertility, train_plain_bpe


def _corpus(n=400, seed=0):
    rng = random.Random(seed)
    words = "the of and to in a is that for it as was with on be by this at from".split()
    nouns = "cat dog house tree river city model token data paper".split()
    out = []
    for _ in range(n):
        out.append(" ".join(rng.choice(words) + " " + rng.choice(nouns) for _ in range(rng.randint(4, 12))) + ".")
    return out


def test_superbpe_extends_vocab_and_lowers_fertility():
    texts = _corpus()
    plain = train_plain_bpe(texts, 300)
    res = extend_with_superwords(plain, texts, 420)
    assert res.n_superword_merges > 0 and res.final_vocab > plain.get_vocab_size()
    spans = [t for t in res.tokenizer.get_vocab() if "Ġ" in t[1:]]  # a space inside a token
    assert spans, "expected superword tokens spanning a word boundary"
    held = _corpus(50, seed=1)
    assert fertility(res.tokenizer, held)["tokens_per_byte"] < fertility(plain, held)["tokens_per_byte"]
    s = held[0]
    assert res.tokenizer.decode(res.tokenizer.encode(s).ids) == s
    assert plain.decode(plain.encode(s).ids) == s


def test_cost_model_and_febpb():
    import math

    from marin_experiments_b200.tokenization.cost_model import ServingCostModel, febpb, fertility_of, fit_scaling

    sm = ServingCostModel()
    assert sm.flops_per_token(200_000) > sm.flops_per_token(100_000)
    long = ServingCostModel(context_len=65536)
    assert long.flops_per_token(128256) > sm.flops_per_token(128256)
    pts = [(c, 2.0 * c ** -0.15 + 0.7) for c in (1e17, 3e17, 1e18, 3e18)]
    fit = fit_scaling(pts)
    assert abs(fit.bpb_at(2e18) - (2.0 * 2e18 ** -0.15 + 0.7)) < 1e-3
    cheaper = febpb(fit, 1e18, 0.8)
    dearer = febpb(fit, 1e18, 1.2)
    assert cheaper < fit.bpb_at(1e18) < dearer
    assert math.isinf(febpb(fit, 1e18, 3.0))
    assert abs(fertility_of(lambda s: list(s.encode()), ["abc", "de"]) - 1.0) < 1e-9
