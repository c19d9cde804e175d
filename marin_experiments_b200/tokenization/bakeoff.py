"""Tokenizer bake-off: arms, domain-weighted fertility, the proxy ladder and the FLOP-equivalent score.

The reference splits this over tokenization/arms.py (registry of arms by design axis),
tokenization/fertility.py (tokens per byte by domain), tokenization/proxy_ladder.py (small
models per arm at a ladder of budgets), tokenization/analysis.py and tokenization/bakeoff.py
(scoring and report) and tokenization/soak_config.py (the n-gram soak run). Here:

* ``TokenizerArm`` / ``ArmRegistry``: an arm is a name, a tokenizer file (``tokenizer.json``, the
  format of the ``tokenizers`` library; no hub access here) or an in-memory tokenizer, its vocabulary
  size (the model's embedding / LM-head width, checked against the tokenizer) and the design axis it
  exercises.
* ``domain_fertility`` / ``weighted_fertility``: tokens per UTF-8 byte per domain and their weighted
  mean (weights normalised; uniform by default).
* ``plan_ladder``: per arm and compute budget, the model the AdamH heuristic sizes for that budget,
  with the arm's vocabulary, its batch and step count: the runs whose (training FLOPs, BPB) points
  feed ``cost_model.fit_scaling``.
* ``score``: per arm the serving cost per byte relative to a reference arm
  (``cost_model.ServingCostModel``), the fitted BPB curve and the FLOP-equivalent BPB at the
  reference budget (``cost_model.febpb``); ``report`` ranks them (lower is better; arms without a
  fit or whose serving alone exceeds the budget last).
* ``SOAK``: the soak run's settings (the hashed n-gram input embedding of ``config.NgramEmbedConfig``
  on the reference geometry).
"""

from __future__ import annotations

import dataclasses
import math
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass, field
from enum import Enum

from ..config import NgramEmbedConfig
from ..optim.heuristic import MoeAdamHHeuristic, build_from_heuristic
from ..utils.flops import compute_flops_per_token
from .cost_model import ServingCostModel, febpb, fit_scaling


class Axis(str, Enum):
    """The design question an arm answers."""

    BASELINE = "baseline"  # an existing vocabulary family
    DERIVED_VOCAB = "derived_vocab"  # a larger vocabulary cut down by merge rank
    TRAINED_BPE = "trained_bpe"  # plain BPE trained on the training mixture
    PRETOK = "pretok"  # pre-tokenisation variants (digits, case)
    SUPERBPE = "superbpe"  # superword merges across whitespace
    NGRAM = "ngram"  # hashed n-gram input embeddings on a base tokenizer
    BYTE = "byte"  # byte-level floor
    UNIGRAM = "unigram"  # Unigram-LM instead of BPE


@dataclass(frozen=True)
class TokenizerArm:
    name: str
    vocab_size: int
    axis: Axis
    path: str | None = None  # a tokenizer.json
    tokenizer: object = field(default=None, compare=False, repr=False)  # or an in-memory tokenizer
    notes: str = ""

    def load(self):
        if self.tokenizer is not None:
            tok = self.tokenizer
        elif self.path is not None:
            from tokenizers import Tokenizer

            tok = Tokenizer.from_file(self.path)
        else:
            raise ValueError(f"arm {self.name!r} has neither a path nor a tokenizer")
        real = tok.get_vocab_size()
        if real != self.vocab_size:
            raise ValueError(f"arm {self.name!r}: declared vocab {self.vocab_size} != tokenizer's {real}")
        return tok

    def encoder(self) -> Callable[[str], Sequence[int]]:
        tok = self.load()
        return lambda text: tok.encode(text).ids


class ArmRegistry:
    def __init__(self, arms: Iterable[TokenizerArm] = ()):
        self._arms: dict[str, TokenizerArm] = {}
        for a in arms:
            self.register(a)

    def register(self, arm: TokenizerArm) -> TokenizerArm:
        if arm.name in self._arms:
            raise KeyError(f"arm {arm.name!r} already registered")
        self._arms[arm.name] = arm
        return arm

    def __getitem__(self, name: str) -> TokenizerArm:
        return self._arms[name]

    def __iter__(self):
        return iter(self._arms.values())

    def __len__(self) -> int:
        return len(self._arms)

    def by_axis(self, axis: Axis) -> list[TokenizerArm]:
        return [a for a in self._arms.values() if a.axis == axis]


def domain_fertility(encode: Callable[[str], Sequence[int]], corpora: dict[str, Iterable[str]]) -> dict[str, dict]:
    """Per domain: tokens, UTF-8 bytes and tokens per byte."""
    out = {}
    for dom, texts in corpora.items():
        n_tok = n_b = 0
        for t in texts:
            n_tok += len(encode(t))
            n_b += len(t.encode("utf-8"))
        out[dom] = {"tokens": n_tok, "bytes": n_b, "tokens_per_byte": n_tok / max(n_b, 1)}
    return out


def weighted_fertility(by_domain: dict[str, dict], weights: dict[str, float] | None = None) -> float:
    doms = list(by_domain)
    w = {d: 1.0 for d in doms} if weights is None else {d: float(weights.get(d, 0.0)) for d in doms}
    tot = sum(w.values())
    if tot <= 0:
        raise ValueError("fertility weights sum to zero over the measured domains")
    return sum(w[d] * by_domain[d]["tokens_per_byte"] for d in doms) / tot


# ------------------------------------------------------------------------------------ proxy ladder
DEFAULT_BUDGETS = (3e17, 1e18, 3e18)  # training FLOPs per proxy run
DEFAULT_HIDDEN = {3e17: 512, 1e18: 768, 3e18: 1024}


@dataclass(frozen=True)
class LadderRun:
    arm: str
    budget: float
    model: object
    batch: int
    steps: int
    tokens: float

    @property
    def run_id(self) -> str:
        return f"bakeoff-{self.arm}-C{self.budget:.0e}-d{self.model.hidden_dim}"


def plan_ladder(arm: TokenizerArm, budgets: Sequence[float] = DEFAULT_BUDGETS,
                hidden_for: dict[float, int] | None = None, seq_len: int = 4096,
                heuristic: MoeAdamHHeuristic | None = None) -> list[LadderRun]:
    """The proxy runs of one arm: the heuristic's model for each budget, at the arm's vocabulary."""
    h = dataclasses.replace(heuristic or MoeAdamHHeuristic(), vocab_size=arm.vocab_size)
    hidden_for = hidden_for or DEFAULT_HIDDEN
    runs = []
    for c in budgets:
        model, _opt, batch, steps = build_from_heuristic(budget=c, hidden_dim=hidden_for[c], heuristic=h,
                                                         seq_len=seq_len)
        tokens = c / (3 * compute_flops_per_token(model))
        runs.append(LadderRun(arm.name, c, model, batch, steps, tokens))
    return runs


# ------------------------------------------------------------------------------------------- score
@dataclass
class ScoredArm:
    name: str
    axis: str
    vocab_size: int
    fertility: float
    serving_flops_per_byte: float
    relative_serving_cost: float
    n_points: int
    febpb: float = math.nan
    bpb_at_reference: float = math.nan


def score(arms: Iterable[TokenizerArm], fertility: dict[str, float], bpb_points: dict[str, list[tuple[float, float]]],
          *, reference: str, serving: ServingCostModel | None = None, serving_ratio: float = 1.0,
          reference_budget: float | None = None) -> list[ScoredArm]:
    """Score every arm against ``reference``. ``fertility``: tokens per byte (weighted); ``bpb_points``:
    (training FLOPs, BPB) of each arm's ladder. The reference training budget is ``reference_budget``
    or the largest FLOPs of the reference arm's ladder."""
    serving = serving or ServingCostModel()
    arms = list(arms)
    by = {a.name: a for a in arms}
    ref = by[reference]
    ref_cost = serving.flops_per_byte(ref.vocab_size, fertility[reference])
    ref_flops = reference_budget or max(f for f, _ in bpb_points[reference])
    rows = []
    for a in arms:
        cost = serving.flops_per_byte(a.vocab_size, fertility[a.name])
        pts = bpb_points.get(a.name, [])
        row = ScoredArm(a.name, a.axis.value, a.vocab_size, fertility[a.name], cost, cost / ref_cost, len(pts))
        if len(pts) >= 3:
            fit = fit_scaling(pts)
            row.bpb_at_reference = fit.bpb_at(ref_flops)
            row.febpb = febpb(fit, ref_flops, row.relative_serving_cost, serving_ratio)
        rows.append(row)
    return sorted(rows, key=lambda r: (not math.isfinite(r.febpb), r.febpb if math.isfinite(r.febpb) else 0.0))


def report(rows: list[ScoredArm]) -> str:
    out = ["| arm | axis | vocab | tokens/byte | rel. serving cost | BPB @ ref budget | feBPB | points |",
           "|---|---|---|---|---|---|---|---|"]
    for r in rows:
        fe = f"{r.febpb:.4f}" if math.isfinite(r.febpb) else ("inf" if r.febpb == math.inf else "-")
        b = f"{r.bpb_at_reference:.4f}" if math.isfinite(r.bpb_at_reference) else "-"
        out.append(f"| {r.name} | {r.axis} | {r.vocab_size} | {r.fertility:.4f} | {r.relative_serving_cost:.3f} | "
                   f"{b} | {fe} | {r.n_points} |")
    return "\n".join(out)


@dataclass(frozen=True)
class SoakParams:
    """The soak run: a long single-arm run with the hashed n-gram input embedding."""

    base_arm: str = "llama3"
    hidden_dim: int = 1536
    budget: float = 1e19
    seq_len: int = 4096
    ngram: NgramEmbedConfig = field(default_factory=NgramEmbedConfig)


SOAK = SoakParams()
