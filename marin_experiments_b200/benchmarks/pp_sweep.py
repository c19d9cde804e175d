"""Pipeline schedule sweep (grug-moe-pp/perf_zb.py:62-221): bubble fraction and makespan of GPipe,
1F1B and ZB-H1 over stage counts and microbatch counts from the schedule simulator, with the
backward split costs of the zero-bubble schedule (B = input gradient, W = weight gradient).

Run: ``python -m marin_experiments_b200.benchmarks.pp_sweep [--json]``.
"""

from __future__ import annotations

import argparse
import json

from marin_experiments_b200.parallel.schedules import SCHEDULES, simulate


def sweep(stages=(2, 4, 8), micro=(4, 8, 16, 32), t_f=1.0, t_b=1.0, t_w=1.0):
    rows = []
    for p in stages:
        for m in micro:
            for name, fn in SCHEDULES.items():
                sched = fn(p, m)
                r = simulate(sched, t_f, t_b, t_w) if name == "zb" else simulate(sched, t_f, t_b + t_w)
                rows.append({"pp": p, "microbatches": m, "schedule": name, "bubble": round(r["bubble"], 4),
                             "makespan": r["makespan"]})
    return rows


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    rows = sweep()
    if a.json:
        print(json.dumps(rows))
    else:
        print("| pp | M | schedule | bubble | makespan |\n|---|---|---|---|---|")
        for r in rows:
            print(f"| {r['pp']} | {r['microbatches']} | {r['schedule']} | {r['bubble']:.3f} | {r['makespan']:.0f} |")
