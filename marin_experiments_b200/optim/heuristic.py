"""Compute-scaling AdamH heuristic for MoE sizing and hyperparameters
(megagpt-speedrun/heuristic.py:79-302).

The fitted coefficients are the reference's (an empirical fit is data, so the numbers have to be
the same): Adam LR ``0.025469 * tokens^-0.2813 * D^-0.3678 * sqrt(tokens_per_batch)`` capped at
0.05; AdamH LR = 13/3 of it; epsilon ``9.676e-18 * sqrt(tokens / tokens_per_batch)``; beta1 0.9062;
beta2 ``clip(0.999^(tpb / 131072), 0.95, 0.9999)``. Sizing from the hidden size: layers
``round(D / (64 + 4 log2 D - 9))``, heads ``D / 128``, 4:1 GQA, expert width ``ceil(D/256) * 128``,
shared expert width D, init std ``0.5 / sqrt(D)``, qk_mult 1.3. The budget convention is
``C = 3 * compute_flops_per_token * tokens`` with a power-of-two batch for ``2^14`` target steps.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from ..config import GrugModelConfig
from ..utils.flops import compute_flops_per_token
from .configs import GrugMoeAdamHConfig

SEQ_LEN = 4096
MIN_BATCH_SIZE = 32
DEFAULT_TARGET_STEPS = 2 ** 14


def round_up_pow2(x: float) -> int:
    return 1 if x <= 1 else 2 ** math.ceil(math.log2(x))


def compute_tokens_and_batch(budget: float, flops_per_token: float, target_steps: int = DEFAULT_TARGET_STEPS,
                             min_batch_size: int = MIN_BATCH_SIZE, seq_len: int = SEQ_LEN) -> tuple[float, int, int]:
    tokens = budget / (3 * flops_per_token)
    batch = max(min_batch_size, round_up_pow2(tokens / (target_steps * seq_len)))
    steps = max(1, round(tokens / (batch * seq_len)))
    return tokens, batch, steps


@dataclass(frozen=True)
class MoeAdamHHeuristic:
    lr_coeff: float = 0.025469
    lr_tokens_exp: float = -0.2813
    lr_dim_exp: float = -0.3678
    adamh_ratio: float = 13 / 3
    epsilon_coeff: float = 9.676e-18
    beta1: float = 0.9062
    beta2_base: float = 0.999
    beta2_reference_tpb: int = 131_072
    max_grad_norm: float = 1.0
    z_loss_weight: float = 1e-4
    min_lr_ratio: float = 0.0
    warmup: float = 0.1
    lr_schedule: str = "linear"
    decay: float | None = None
    vocab_size: int = 128_256
    hidden_head_ratio: int = 128
    gqa_ratio: int | None = 4
    base_hidden_layer_ratio: int = 64
    layer_scaling_factor: float = 4.0
    layer_formula_offset: int = 9
    max_learning_rate: float = 0.05
    min_beta2: float = 0.95
    max_beta2: float = 0.9999

    def adam_lr(self, tokens_per_batch: int, tokens: float, hidden: int) -> float:
        lr = self.lr_coeff * tokens ** self.lr_tokens_exp * hidden ** self.lr_dim_exp * math.sqrt(tokens_per_batch)
        return min(self.max_learning_rate, lr)

    def adamh_lr(self, tokens_per_batch: int, tokens: float, hidden: int) -> float:
        return min(self.max_learning_rate, self.adamh_ratio * self.adam_lr(tokens_per_batch, tokens, hidden))

    def epsilon(self, tokens_per_batch: int, tokens: float) -> float:
        return self.epsilon_coeff * math.sqrt(tokens / tokens_per_batch)

    def beta2(self, tokens_per_batch: int) -> float:
        b = self.beta2_base ** (tokens_per_batch / self.beta2_reference_tpb)
        return max(self.min_beta2, min(self.max_beta2, b))

    def build_optimizer_config(self, batch_size: int, tokens: float, hidden: int,
                               seq_len: int = SEQ_LEN) -> GrugMoeAdamHConfig:
        tpb = batch_size * seq_len
        return GrugMoeAdamHConfig(learning_rate=self.adamh_lr(tpb, tokens, hidden),
                                  adam_lr=self.adam_lr(tpb, tokens, hidden), min_lr_ratio=self.min_lr_ratio,
                                  warmup=self.warmup, beta1=self.beta1, beta2=self.beta2(tpb),
                                  epsilon=self.epsilon(tpb, tokens), max_grad_norm=self.max_grad_norm,
                                  lr_schedule=self.lr_schedule, decay=self.decay)

    def num_layers(self, hidden: int) -> int:
        return round(hidden / (self.base_hidden_layer_ratio + math.log2(hidden) * self.layer_scaling_factor
                               - self.layer_formula_offset))

    @staticmethod
    def kv_heads(num_heads: int, gqa_ratio: int | None) -> int:
        if gqa_ratio is None:
            return num_heads
        for k in range(num_heads // gqa_ratio, 0, -1):
            if num_heads % k == 0:
                return k
        return 1

    def build_model_config(self, hidden: int, seq_len: int = SEQ_LEN, *, num_experts: int = 64,
                           num_experts_per_token: int = 4, adaptive_routing: bool = False,
                           min_experts_per_token: int = 0, sparsity_loss_coef: float = 0.0,
                           sparsity_temp: float = 1.0, embed_dim: int | None = None) -> GrugModelConfig:
        if hidden % self.hidden_head_ratio:
            raise ValueError(f"hidden_size ({hidden}) must be divisible by {self.hidden_head_ratio}")
        heads = max(1, hidden // self.hidden_head_ratio)
        return GrugModelConfig(vocab_size=self.vocab_size, hidden_dim=hidden, embed_dim=embed_dim,
                               intermediate_dim=math.ceil(hidden / 2 / 128) * 128,
                               shared_expert_intermediate_dim=hidden, num_experts=num_experts,
                               num_experts_per_token=num_experts_per_token, adaptive_routing=adaptive_routing,
                               min_experts_per_token=min_experts_per_token, sparsity_loss_coef=sparsity_loss_coef,
                               sparsity_temp=sparsity_temp, num_layers=self.num_layers(hidden), num_heads=heads,
                               num_kv_heads=self.kv_heads(heads, self.gqa_ratio), max_seq_len=seq_len,
                               sliding_window=seq_len, initializer_std=0.5 / math.sqrt(hidden), qk_mult=1.3)


def build_from_heuristic(*, budget: float, hidden_dim: int, heuristic: MoeAdamHHeuristic | None = None,
                         target_steps: int = DEFAULT_TARGET_STEPS, min_batch_size: int = MIN_BATCH_SIZE,
                         seq_len: int = SEQ_LEN, batch_size: int | None = None, model_overrides: dict | None = None):
    """(model config, optimizer config, batch size, steps) for a compute budget. ``batch_size`` pins
    the batch exactly (memory-capped runs) and derives the step count from it."""
    h = heuristic or MoeAdamHHeuristic()
    model = h.build_model_config(hidden_dim, seq_len=seq_len, **(model_overrides or {}))
    tokens, batch, steps = compute_tokens_and_batch(budget, compute_flops_per_token(model), target_steps,
                                                    min_batch_size, seq_len)
    if batch_size is not None:
        batch = int(batch_size)
        steps = max(1, round(tokens / (batch * seq_len)))
    return model, h.build_optimizer_config(batch, tokens, hidden_dim, seq_len=seq_len), batch, steps
