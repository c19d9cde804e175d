"""Tokenizer bake-off: arms registry, weighted fertility, proxy-ladder plan, feBPB scoring."""

import math

import pytest

from marin_experiments_b200.tokenization import bakeoff as bo
from marin_experiments_b200.tokenization.superbpe import train_plain_bpe

TEXT = ["the quick brown fox jumps over the lazy dog " * 4, "def f(x):\n    return x * 2 + 1\n" * 4,
        "numbers 12345 67890 and more numbers 424242 " * 4] * 8
CORPORA = {"web": TEXT[0::3], "code": TEXT[1::3], "math": TEXT[2::3]}


@pytest.fixture(scope="module")
def arms(tmp_path_factory):
    small = train_plain_bpe(TEXT, 300)
    big = train_plain_bpe(TEXT, 420)
    path = str(tmp_path_factory.mktemp("tok") / "big.json")
    big.save(path)
    reg = bo.ArmRegistry([bo.TokenizerArm("bpe300", small.get_vocab_size(), bo.Axis.TRAINED_BPE, tokenizer=small),
                          bo.TokenizerArm("bpe420", big.get_vocab_size(), bo.Axis.DERIVED_VOCAB, path=path)])
    return reg


def test_registry_and_fertility(arms):
    assert len(arms) == 2 and [a.name for a in arms.by_axis(bo.Axis.DERIVED_VOCAB)] == ["bpe420"]
    with pytest.raises(KeyError):
        arms.register(arms["bpe300"])
    with pytest.raises(ValueError):
        bo.TokenizerArm("bad", 12345, bo.Axis.BYTE, tokenizer=arms["bpe300"].load()).load()
    f_small = bo.domain_fertility(arms["bpe300"].encoder(), CORPORA)
    f_big = bo.domain_fertility(arms["bpe420"].encoder(), CORPORA)
    assert set(f_small) == {"web", "code", "math"} and f_small["web"]["bytes"] > 0
    w_small, w_big = bo.weighted_fertility(f_small), bo.weighted_fertility(f_big)
    assert w_big <= w_small  # a larger vocabulary of the same trainer never needs more tokens here
    only_code = bo.weighted_fertility(f_small, {"code": 1.0})
    assert only_code == f_small["code"]["tokens_per_byte"]
    with pytest.raises(ValueError):
        bo.weighted_fertility(f_small, {"none": 1.0})


def test_ladder_plan(arms):
    runs = bo.plan_ladder(arms["bpe420"])
    assert [r.budget for r in runs] == list(bo.DEFAULT_BUDGETS)
    assert all(r.model.vocab_size == arms["bpe420"].vocab_size for r in runs)
    assert [r.model.hidden_dim for r in runs] == [512, 768, 1024]
    assert runs[0].tokens < runs[-1].tokens and runs[0].steps >= 1 and "bakeoff-bpe420-C3e+17" in runs[0].run_id


def test_score_ranks_by_febpb(arms):
    fert = {"bpe300": 0.30, "bpe420": 0.25}
    pts = {"bpe300": [(1e17, 1.30), (3e17, 1.20), (1e18, 1.12), (3e18, 1.07)],
           "bpe420": [(1e17, 1.29), (3e17, 1.19), (1e18, 1.11), (3e18, 1.06)]}
    rows = bo.score(arms, fert, pts, reference="bpe300")
    by = {r.name: r for r in rows}
    assert by["bpe300"].relative_serving_cost == 1.0 and by["bpe420"].relative_serving_cost < 1.0
    assert rows[0].name == "bpe420" and rows[0].febpb < by["bpe300"].febpb
    # the reference arm's feBPB is its own fitted BPB at the reference budget
    assert math.isclose(by["bpe300"].febpb, by["bpe300"].bpb_at_reference, rel_tol=1e-9)
    # an arm without a ladder is listed last, unscored
    rows2 = bo.score(arms, fert, {"bpe300": pts["bpe300"]}, reference="bpe300")
    assert rows2[-1].name == "bpe420" and math.isnan(rows2[-1].febpb) and rows2[-1].n_points == 0
    text = bo.report(rows2)
    assert text.count("\n") == 3 and "| bpe420 |" in text
    assert bo.SOAK.ngram.orders == (2, 3, 4)
