"""Concrete optimizer configs.

* ``GrugMoeAdamHConfig`` ("grug_moe_adamh_v2", megagpt-speedrun/optimizer.py:14-92): three groups --
  ``adamh`` (2-D matrices, ``learning_rate``), ``adamh_expert`` (routed + shared expert and dense
  MLP weights, ``expert_lr`` or ``learning_rate``), ``adam`` (embeddings, router, attention gates,
  1-D params, ``adam_lr``) -- each clipped by its own global norm.
* ``AdamConfig`` ("adam"): AdamW with decoupled weight decay on >= 2-D params (levanter
  AdamConfig, used by tiny-stories/launch.py:229-236).
* ``MuonConfig`` ("muon"): Newton-Schulz orthogonalised momentum on 2-D / per-expert matrices,
  AdamW on the rest (levanter GrugMuonConfig; NS in megagpt-speedrun/async_pipeline.py:371-403).
"""

from __future__ import annotations

from dataclasses import dataclass

from .base import OptimizerConfig, grug_group_of, register


@register("grug_moe_adamh_v2")
@dataclass(frozen=True)
class GrugMoeAdamHConfig(OptimizerConfig):
    learning_rate: float = 0.02
    adam_lr: float = 6e-4
    expert_lr: float | None = None
    lr_schedule: str = "linear"
    warmup: float = 0.1
    min_lr_ratio: float = 0.0

    def groups(self, store):
        out = {
            "adamh": {"kind": "adamh", "lr": self.learning_rate, "infos": [], "wd": 0.0},
            "adamh_expert": {"kind": "adamh", "lr": self.expert_lr if self.expert_lr is not None
                             else self.learning_rate, "infos": [], "wd": 0.0},
            "adam": {"kind": "adam", "lr": self.adam_lr, "infos": [], "wd": 0.0},
        }
        for info in store.infos:
            if not info.trainable:
                continue
            out[grug_group_of(info.name, info.ndim)]["infos"].append(info)
        return out


@register("adam")
@dataclass(frozen=True)
class AdamConfig(OptimizerConfig):
    learning_rate: float = 3e-4
    weight_decay: float = 0.0
    beta2: float = 0.999

    def groups(self, store):
        decay = {"kind": "adam", "lr": self.learning_rate, "infos": [], "wd": self.weight_decay}
        nodecay = {"kind": "adam", "lr": self.learning_rate, "infos": [], "wd": 0.0}
        for info in store.infos:
            if not info.trainable:
                continue
            (decay if info.ndim >= 2 else nodecay)["infos"].append(info)
        return {"decay": decay, "no_decay": nodecay}


@register("muon")
@dataclass(frozen=True)
class MuonConfig(OptimizerConfig):
    learning_rate: float = 0.02
    adam_lr: float = 6e-4
    momentum: float = 0.95
    ns_steps: int = 5
    nesterov: bool = True

    def groups(self, store):
        muon = {"kind": "muon", "lr": self.learning_rate, "infos": [], "wd": self.weight_decay}
        adam = {"kind": "adam", "lr": self.adam_lr, "infos": [], "wd": 0.0}
        for info in store.infos:
            if not info.trainable:
                continue
            g = grug_group_of(info.name, info.ndim)
            (muon if g != "adam" else adam)["infos"].append(info)
        return {"muon": muon, "adam": adam}
