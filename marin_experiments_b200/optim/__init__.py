"""Optimizers: AdamH / Adam(W) / Muon over the flat parameter store, and the delayed-gradient wrapper."""

from .base import OPTIMIZER_REGISTRY, OptimizerConfig, grug_group_of, lr_schedule_fn, register  # noqa: F401
from .configs import AdamConfig, GrugMoeAdamHConfig, MuonConfig  # noqa: F401
from .delayed import (  # noqa: F401
    CORRECTORS,
    DelayedGrugMoeAdamHConfig,
    DelayedGrugMuonConfig,
    DelayedOptimizer,
    grug_stage_tau,
)
from .fused import FusedOptimizer  # noqa: F401
