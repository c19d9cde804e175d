"""Optimizer config base, registry and learning-rate schedules.

``OptimizerConfig`` mirrors the levanter fields the reference configures
(megagpt-speedrun/launch.py:293-372, tiny-stories/launch.py:229-236): ``learning_rate``,
``weight_decay``, ``warmup`` (fraction of steps if < 1, else steps), ``decay`` (fraction or steps of the
final decay phase; ``None`` = everything after warmup), ``min_lr_ratio``, ``lr_schedule`` in
{constant, linear, cosine, inv_sqrt}, ``rewarmup`` and ``max_grad_norm``. Subclasses register a
name with ``@register("grug_moe_adamh_v2")`` and build a ``FusedOptimizer`` over a ``ParamStore``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

OPTIMIZER_REGISTRY: dict[str, type] = {}


def register(name: str):
    def deco(cls):
        OPTIMIZER_REGISTRY[name] = cls
        cls.registry_name = name
        return cls

    return deco


def lr_schedule_fn(peak: float, num_steps: int, *, warmup: float = 0.0, decay: float | None = None,
                   min_lr_ratio: float = 0.0, schedule: str = "linear", rewarmup: float = 0.0):
    """Learning rate as a function of the step (warmup -> stable -> decay, WSD when ``decay`` < all)."""
    n = max(1, int(num_steps))
    w = int(round(warmup * n)) if warmup < 1 else int(warmup)
    if decay is None:
        d = n - w
    else:
        d = int(round(decay * n)) if decay < 1 else int(decay)
    d = max(0, min(d, n - w))
    stable = n - w - d
    rw = int(round(rewarmup * n)) if rewarmup < 1 else int(rewarmup)
    lo = peak * min_lr_ratio

    def lr(step: int) -> float:
        if rw > 0 and step < rw:
            return lo + (peak - lo) * (step + 1) / rw
        if step < w:
            return peak * (step + 1) / w
        if schedule == "constant" or step < w + stable:
            if schedule == "inv_sqrt" and step >= w:
                return peak * math.sqrt(max(w, 1) / (step + 1))
            return peak
        p = min(1.0, (step - w - stable) / max(1, d))
        if schedule == "linear":
            return peak - (peak - lo) * p
        if schedule == "cosine":
            return lo + (peak - lo) * 0.5 * (1 + math.cos(math.pi * p))
        if schedule == "inv_sqrt":
            return peak * math.sqrt(max(w, 1) / (step + 1))
        raise ValueError(f"unknown lr_schedule {schedule}")

    return lr


@dataclass(frozen=True)
class OptimizerConfig:
    learning_rate: float = 6e-4
    weight_decay: float = 0.0
    beta1: float = 0.9
    beta2: float = 0.95
    epsilon: float = 1e-8
    max_grad_norm: float | None = 1.0
    warmup: float = 0.01
    decay: float | None = None
    min_lr_ratio: float = 0.1
    lr_schedule: str = "cosine"
    rewarmup: float = 0.0

    def lr_scheduler(self, num_train_steps: int, override_lr: float | None = None):
        peak = self.learning_rate if override_lr is None else override_lr
        return lr_schedule_fn(peak, num_train_steps, warmup=self.warmup, decay=self.decay,
                              min_lr_ratio=self.min_lr_ratio, schedule=self.lr_schedule, rewarmup=self.rewarmup)

    def groups(self, store) -> dict[str, dict]:
        """name -> {"kind": "adam"|"adamh", "lr_fn": step -> lr, "infos": [...], "wd": float}."""
        raise NotImplementedError

    def build(self, store, num_train_steps: int):
        from .fused import FusedOptimizer

        return FusedOptimizer(store, self, num_train_steps)


def grug_group_of(name: str, ndim: int) -> str:
    """Parameter-group rule of ``grug_moe_adamh_v2`` (megagpt-speedrun/optimizer.py:80-92)."""
    p = name.lower()
    if "token_embed" in p or "ngram_table" in p:
        return "adam"
    # zero-initialised modulation / bias parameters of the looped model: a scale-invariant step
    # cannot move a zero matrix (reentrant/optimizer.py routes them to Adam too)
    if "film_" in p or "depth_bias" in p or "halt_head" in p:
        return "adam"
    if "router_bias" in p or "attn_gate" in p or ".router" in p or p.startswith("router"):
        return "adam"
    if ".mlp.w_" in p or ".shared.w_" in p or ".mlp.expert_mlp.w_" in p:
        return "adamh_expert"
    if ndim >= 2:
        return "adamh"
    return "adam"
