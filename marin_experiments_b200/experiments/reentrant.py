"""Re-entrant (looped) grug MoE experiment series (reentrant/launch.py): every experiment shares the
E0 baseline's optimizer, batch, step count, data and evaluation, so only the architecture differs
and the curves compare directly. ``GRUG_EXPERIMENT`` selects experiments (comma-separated, default
``e0``); ``CONSISTENCY_WEIGHT``, ``ANYTIME_WEIGHT``, ``PONDER_KL`` and ``PONDER_PRIOR`` tune the
regularised variants.

* e0: the d512 grug MoE from the AdamH compute heuristic (budget 2.19e17 FLOPs, 2^14 target steps);
* e1: 1 prelude + 1 weight-tied core looped 4 times + 1 coda (effective depth 6, three blocks);
* e2: e1 + per-iteration FiLM on the core;
* e3: e1 with the loop count drawn per step from {2, 4, 8} (test-time depth scaling);
* e4: e3 + anytime deep supervision (a CE read off the head after every core iteration);
* e5: e3 + the core-consistency penalty;
* e6: e3 + depth-conditioned routing (a learned router bias per iteration and core layer);
* e64: e6 + anytime supervision;  e7: e3 + PonderNet halting.

Run: ``GRUG_EXPERIMENT=e1,e3 python -m marin_experiments_b200.experiments.reentrant [--prefix D]
[--dry_run]``; ``train.eval.evaluate_at_depths`` sweeps a trained checkpoint over loop counts.
"""

from __future__ import annotations

import dataclasses
import os

from ..config import DataConfig, GrugEvalConfig, GrugTrainerConfig
from ..executor import ExecutorStep, executor_main, this_output_path, versioned
from ..models.looped import LoopedConfig
from ..optim.heuristic import build_from_heuristic
from .common import GrugLaunchConfig, run_inline

BUDGET, HIDDEN, TARGET_STEPS = 2.19e17, 512, 2 ** 14


def _f(key: str, default: float) -> float:
    raw = os.environ.get(key, "")
    return float(raw) if raw else default


def experiments() -> dict[str, tuple[object, LoopedConfig | None]]:
    """name -> (model config, looped config or None for the plain baseline)."""
    base, _, _, _ = build_from_heuristic(budget=BUDGET, hidden_dim=HIDDEN, target_steps=TARGET_STEPS)
    core = dataclasses.replace(base, num_layers=3)
    e1 = LoopedConfig(model=core, num_prelude_layers=1, num_coda_layers=1, recurrence_steps=4)
    e3 = dataclasses.replace(e1, randomize_recurrence=True, recurrence_choices=(2, 4, 8))
    e6 = dataclasses.replace(e3, depth_conditioned_routing=True)
    anytime = dict(anytime_supervision=True, anytime_supervision_weight=_f("ANYTIME_WEIGHT", 1.0))
    looped = {
        "e1": e1,
        "e2": dataclasses.replace(e1, iteration_film=True),
        "e3": e3,
        "e4": dataclasses.replace(e3, **anytime),
        "e5": dataclasses.replace(e3, core_consistency_weight=_f("CONSISTENCY_WEIGHT", 1.0)),
        "e6": e6,
        "e64": dataclasses.replace(e6, **anytime),
        "e7": dataclasses.replace(e3, ponder_halting=True, ponder_kl_weight=_f("PONDER_KL", 0.01),
                                  ponder_prior_lambda=_f("PONDER_PRIOR", 0.2)),
    }
    return {"e0": (base, None), **{k: (core, v) for k, v in looped.items()}}


def build_steps(selected: list[str] | None = None, data: DataConfig | None = None) -> list[ExecutorStep]:
    base, opt, batch, steps = build_from_heuristic(budget=BUDGET, hidden_dim=HIDDEN, target_steps=TARGET_STEPS)
    exps = experiments()
    names = selected or [x for x in os.environ.get("GRUG_EXPERIMENT", "e0").split(",") if x]
    unknown = [n for n in names if n not in exps]
    if unknown:
        raise KeyError(f"unknown experiment(s) {unknown}; known: {sorted(exps)}")
    data = data or DataConfig(source="synthetic", seed=0)
    out = []
    for n in names:
        model, lc = exps[n]
        run_id = os.environ.get("GRUG_RUN_ID") or f"reentrant_{n}_d{HIDDEN}"
        out.append(ExecutorStep(name=f"grug/reentrant_{n}", fn=run_inline, config=GrugLaunchConfig(
            model=versioned(model), looped=versioned(lc), data=data, output_path=this_output_path(), run_id=run_id,
            steps=versioned(steps), batch_size=versioned(batch), seed=versioned(0),
            mp=versioned("params=float32,compute=bfloat16,output=bfloat16"), optimizer=versioned(opt),
            grug_trainer=versioned(GrugTrainerConfig(z_loss_weight=1e-4, ema_beta=None, log_every=1)),
            eval=versioned(GrugEvalConfig(eval_batch_size=512, steps_per_eval=1000, max_eval_batches=8,
                                          eval_current=True, eval_ema=False)))))
    return out


def main(argv=None):
    return executor_main(build_steps(), description="re-entrant grug MoE experiments", argv=argv)


if __name__ == "__main__":
    main()
