"""Delayed-gradient launcher: ``GRUG_*`` arms for training under simulated pipeline staleness.

The reference's delayed-gradient template selects its arms with ``GRUG_*`` environment variables
(delayed-gradient-pp/launch.py:12-26, configs built at :133-192). The same arms here:

``GRUG_OPT`` muon | adamh (default muon); ``GRUG_TAU`` uniform delay in steps (default 0, ignored when
``GRUG_STAGES`` > 0); ``GRUG_STAGES`` pipeline stages of the per-stage delay profile
(``optim.delayed.grug_stage_tau``; default 0 = uniform); ``GRUG_CORRECTOR`` none | dc_asgd |
dc_asgd_ema | weight_pred | lr_damp | wp_preorth | wp_cautious | wp_trust | wp_confidence;
``GRUG_DC_LAMBDA`` (1.0), ``GRUG_PRED_SCALE`` (1.0), ``GRUG_PRED_BETA`` (0.95), ``GRUG_TRUST`` (0.01),
``GRUG_LR_DAMP`` (1.0); ``GRUG_STEPS`` (3000), ``GRUG_SEED`` (0), ``GRUG_HIDDEN`` (512), ``GRUG_BUDGET``
(2.19e17, the heuristic's sizing and learning-rate budget), ``GRUG_SEQ`` (4096), ``GRUG_BATCH``
(the heuristic's batch by default), ``GRUG_GROUP`` (a tag carried in the run id). Data is synthetic.

Usage: ``GRUG_OPT=muon GRUG_TAU=8 GRUG_CORRECTOR=dc_asgd_ema python -m
marin_experiments_b200.experiments.delayed_gradient [--dry_run]``.
"""

from __future__ import annotations

import dataclasses
import os
import sys

from ..config import DataConfig, GrugTrainerConfig
from ..executor import ExecutorStep, executor_main, this_output_path, versioned
from ..optim.delayed import DelayedGrugMoeAdamHConfig, DelayedGrugMuonConfig
from ..optim.heuristic import build_from_heuristic
from .common import GrugLaunchConfig, run_inline

CORRECTORS = ("none", "dc_asgd", "dc_asgd_ema", "weight_pred", "lr_damp", "wp_preorth", "wp_cautious", "wp_trust",
              "wp_confidence")


def _env(env, key: str, default: str) -> str:
    v = (env if env is not None else os.environ).get(key)
    return default if v in (None, "") else v


def make_launch(env=None) -> tuple[GrugLaunchConfig, str]:
    opt_kind = _env(env, "GRUG_OPT", "muon")
    if opt_kind not in ("muon", "adamh"):
        raise ValueError(f"GRUG_OPT must be muon or adamh, got {opt_kind!r}")
    corrector = _env(env, "GRUG_CORRECTOR", "none")
    if corrector not in CORRECTORS:
        raise ValueError(f"GRUG_CORRECTOR must be one of {CORRECTORS}, got {corrector!r}")
    stages = int(_env(env, "GRUG_STAGES", "0"))
    tau = 0 if stages > 0 else int(_env(env, "GRUG_TAU", "0"))
    hidden = int(_env(env, "GRUG_HIDDEN", "512"))
    budget = float(_env(env, "GRUG_BUDGET", "2.19e17"))
    seq = int(_env(env, "GRUG_SEQ", "4096"))
    seed = int(_env(env, "GRUG_SEED", "0"))
    model, adamh, batch, _ = build_from_heuristic(budget=budget, hidden_dim=hidden, seq_len=seq)
    batch = int(_env(env, "GRUG_BATCH", str(batch)))
    steps = int(_env(env, "GRUG_STEPS", "3000"))
    delay = dict(tau=tau, corrector=corrector, dc_lambda=float(_env(env, "GRUG_DC_LAMBDA", "1.0")),
                 pred_scale=float(_env(env, "GRUG_PRED_SCALE", "1.0")),
                 pred_beta=float(_env(env, "GRUG_PRED_BETA", "0.95")), trust=float(_env(env, "GRUG_TRUST", "0.01")),
                 lr_damp=float(_env(env, "GRUG_LR_DAMP", "1.0")), num_stages=stages, num_layers=model.num_layers)
    if opt_kind == "adamh":
        opt = DelayedGrugMoeAdamHConfig(**{f.name: getattr(adamh, f.name) for f in dataclasses.fields(adamh)}, **delay)
    else:  # Muon on the matrices, Adam at the heuristic's learning rate on the rest
        opt = DelayedGrugMuonConfig(adam_lr=adamh.adam_lr, warmup=adamh.warmup, lr_schedule=adamh.lr_schedule,
                                    max_grad_norm=adamh.max_grad_norm, **delay)
    group = _env(env, "GRUG_GROUP", "delay-pp-batch1")
    delay_tag = f"S{stages}" if stages > 0 else f"tau{tau}"
    run_id = f"{group}-{opt_kind}-{delay_tag}-{corrector}-d{hidden}-s{seed}"
    launch = GrugLaunchConfig(
        model=versioned(model), data=DataConfig(source="synthetic", seq_len=seq, seed=seed),
        output_path=this_output_path(), run_id=run_id, steps=versioned(steps), batch_size=versioned(batch),
        seed=versioned(seed), optimizer=versioned(opt),
        grug_trainer=versioned(GrugTrainerConfig(z_loss_weight=1e-4, ema_beta=None, log_every=1)))
    arm = (f"[arm] {run_id}  opt={opt_kind} tau={tau} stages={stages} corrector={corrector} D={hidden} "
           f"layers={model.num_layers} seq={seq} batch={batch} steps={steps} budget={budget:g}")
    return launch, arm


def make_step(env=None) -> ExecutorStep:
    launch, arm = make_launch(env)
    print(arm, flush=True)
    return ExecutorStep(name=f"grug/delayed/{launch.run_id}", fn=run_inline, config=launch)


def main(argv=None):
    return executor_main([make_step()], description="Grug training under delayed gradients (GRUG_* arms).",
                         argv=argv)


if __name__ == "__main__":
    main(sys.argv[1:])
