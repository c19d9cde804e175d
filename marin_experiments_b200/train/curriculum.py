"""Active-expert (k) curriculum (megagpt-speedrun/train.py:335-383,696-719).

A schedule is ``((k0, end0), (k1, end1), ...)``: routed top-k ``k_i`` until step ``end_i``. The
model starts at ``k0`` and is widened in place at each boundary; the weights are untouched (every
expert already exists -- only the number each token is routed to changes), so no state has to be
transplanted. ``parse_curriculum("2:0.5,4:0.5", steps)`` reads the launcher's ``k:fraction`` form.
"""

from __future__ import annotations

import dataclasses


def parse_curriculum(spec: str, num_steps: int) -> tuple[tuple[int, int], ...]:
    ks, fracs = [], []
    for part in spec.split(","):
        k, f = part.split(":")
        ks.append(int(k))
        fracs.append(float(f))
    ends, acc = [], 0.0
    for i, f in enumerate(fracs):
        acc += f
        ends.append(num_steps if i == len(fracs) - 1 else max(1, round(acc * num_steps)))
    return tuple(zip(ks, ends))


def active_k_at(schedule, step: int) -> int:
    for k, end in schedule:
        if step < end:
            return k
    return schedule[-1][0]


def set_active_k(model, k: int) -> bool:
    """Route every MoE layer of ``model`` to ``k`` experts; returns True when anything changed."""
    changed = False
    for mod in model.modules():
        cfg = getattr(mod, "cfg", None)
        if cfg is not None and getattr(cfg, "num_experts", 0) > 0 and cfg.num_experts_per_token != k:
            if k > cfg.num_experts:
                raise ValueError(f"k={k} exceeds num_experts={cfg.num_experts}")
            mod.cfg = dataclasses.replace(cfg, num_experts_per_token=k,
                                          min_experts_per_token=min(cfg.min_experts_per_token, k))
            changed = True
    return changed


class KCurriculumHook:
    """Trainer pre-step hook: applies the schedule's k before each step."""

    def __init__(self, schedule):
        self.schedule = tuple(schedule)
        self.current = None

    def before_step(self, trainer) -> None:
        k = active_k_at(self.schedule, trainer.step)
        if k != self.current:
            set_active_k(trainer.model, k)
            trainer.mcfg = dataclasses.replace(trainer.mcfg, num_experts_per_token=k,
                                               min_experts_per_token=min(trainer.mcfg.min_experts_per_token, k))
            self.current = k
