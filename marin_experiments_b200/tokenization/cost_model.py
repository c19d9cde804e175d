"""Tokenizer bake-off pricing: serving cost per byte and FLOP-equivalent BPB
(tokenization/cost_model.py:37-339).

Measurements (proxy training FLOPs, BPB, fertility in tokens/byte) are kept separate from the
deployment model that prices them (``ServingCostModel``): the forward FLOPs per served token of a
target model at a serving context, with local/global attention (one global layer in
``global_layer_period``, the rest over ``attention_window``) and the LM head at the arm's vocabulary.
Per byte, serving cost is ``fertility * flops_per_token``. ``fit_scaling`` fits
``BPB(C) = a C^-b + c`` to an arm's (training FLOPs, BPB) points; ``febpb`` re-invests an arm's
serving savings (relative to a reference tokenizer) into training under a fixed lifetime budget
``B = C_ref (1 + serving_ratio)`` and reads the fitted curve there (an arm whose serving alone
exceeds the budget scores ``inf``).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass, field

from ..config import GrugModelConfig


def _target() -> GrugModelConfig:
    return GrugModelConfig(vocab_size=128256, hidden_dim=2048, intermediate_dim=1024,
                           shared_expert_intermediate_dim=2048, num_experts=64, num_experts_per_token=4,
                           num_layers=24, num_heads=16, num_kv_heads=4, head_dim=128, max_seq_len=16384,
                           sliding_window=16384)


def attention_flops_per_token(cfg: GrugModelConfig, positions: int) -> float:
    """Forward attention FLOPs of one token attending ``positions`` keys (scores + softmax + values)."""
    h, hd = cfg.num_heads, cfg.inferred_head_dim
    return positions * (4 * h * hd + 3 * h)


@dataclass(frozen=True)
class ServingCostModel:
    model: GrugModelConfig = field(default_factory=_target)
    context_len: int = 16_384
    attention_window: int = 4_096
    global_layer_period: int = 6
    speed_factor: float = 1.0

    def attention_per_token(self) -> float:
        g = 1.0 / self.global_layer_period
        w = min(self.attention_window, self.context_len)
        return g * attention_flops_per_token(self.model, self.context_len) + (1 - g) * attention_flops_per_token(self.model, w)

    def flops_per_token(self, vocab_size: int, include_lm_head: bool = True) -> float:
        m = self.model
        d, hd = m.hidden_dim, m.inferred_head_dim
        mlp = 2 * 3 * d * m.intermediate_dim * m.num_experts_per_token + 2 * 3 * d * m.shared_expert_intermediate_dim
        if m.num_experts > 1:
            mlp += 2 * d * m.num_experts
        proj = 2 * d * (m.num_heads * hd + 2 * m.num_kv_heads * hd) + 2 * m.num_heads * hd * d
        head = 2 * d * vocab_size if include_lm_head else 0
        return self.speed_factor * (m.num_layers * (mlp + proj + self.attention_per_token()) + head)

    def flops_per_byte(self, vocab_size: int, fertility: float) -> float:
        return fertility * self.flops_per_token(vocab_size)


@dataclass(frozen=True)
class ScalingFit:
    a: float
    b: float
    c: float

    def bpb_at(self, flops: float) -> float:
        return self.a * flops ** (-self.b) + self.c


def fit_scaling(points: Sequence[tuple[float, float]]) -> ScalingFit:
    """Least-squares fit of ``BPB = a C^-b + c`` (b in (0, 1)), from >= 3 points."""
    import numpy as np
    from scipy.optimize import curve_fit

    if len(points) < 3:
        raise ValueError("need >= 3 (flops, bpb) points")
    c_arr = np.array([p[0] for p in points], dtype=np.float64)
    y = np.array([p[1] for p in points], dtype=np.float64)
    scale = float(np.exp(np.mean(np.log(c_arr))))
    x = c_arr / scale

    def f(x, a, b, c):
        return a * x ** (-b) + c

    p0 = (max(y.max() - y.min(), 1e-3), 0.2, max(y.min() - 0.1, 0.0))
    (a, b, c), _ = curve_fit(f, x, y, p0=p0, bounds=([0, 1e-4, -10], [np.inf, 1.0, 10]), maxfev=20000)
    return ScalingFit(a=float(a) * scale ** float(b), b=float(b), c=float(c))


def febpb(fit: ScalingFit, reference_train_flops: float, relative_serving_cost: float,
          serving_ratio: float = 1.0) -> float:
    train = reference_train_flops * (1.0 + serving_ratio * (1.0 - relative_serving_cost))
    return math.inf if train <= 0 else fit.bpb_at(train)


def fertility_of(encode: Callable[[str], Sequence[int]], corpus: Iterable[str]) -> float:
    """Tokens per UTF-8 byte of ``corpus`` under ``encode``."""
    n_tok = n_b = 0
    for t in corpus:
        n_tok += len(encode(t))
        n_b += len(t.encode("utf-8"))
    return n_tok / max(n_b, 1)
