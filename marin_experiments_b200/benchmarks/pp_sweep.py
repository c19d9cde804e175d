"""Pipeline schedule sweep (grug-moe-pp/perf_zb.py:62-221).

* simulated: bubble fraction and makespan of GPipe, 1F1B and ZB-H1 over stage counts and
  microbatch counts from the schedule simulator, with the backward split costs of the zero-bubble
  schedule (B = input gradient, W = weight gradient);
* measured (``--gpus N``): every schedule (and the async no-flush mode) x stage transport (``p2p``
  NCCL isend / irecv, ``null`` = no traffic, the compute-only reference) timed on N GPUs of this
  node through ``bench.py --config pp`` (device-timed, max over ranks), so the measured cost of the
  transport and of the bubble sit next to the simulated bubble.

Run: ``python -m marin_experiments_b200.benchmarks.pp_sweep [--json] [--gpus N --layers L --steps K]``.
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


def measure(gpus: int, *, schedules=("gpipe", "1f1b", "zb", "async"), transports=("p2p", "null"), layers=None,
            steps: int = 2, warmup: int = 2, port: int = 29650, timeout_s: float = 900.0) -> list[dict]:
    """Time every schedule x transport with ``bench.py --config pp`` on ``gpus`` GPUs."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    rows = []
    for sched in schedules:
        for xport in transports:
            port += 1
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
                   "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(root, "bench.py"),
                   "--gpus", str(gpus), "--config", "pp", "--pp-schedule", sched, "--steps", str(steps),
                   "--warmup", str(warmup), "--no-e2e"]
            if layers:
                cmd += ["--layers", str(layers)]
            env = dict(os.environ, SP_PP_TRANSPORT=xport)
            try:
                out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout_s, cwd=root)
                line = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
                d = json.loads(line[-1]) if line else {}
            except subprocess.TimeoutExpired:
                d = {}
            rows.append({"schedule": sched, "transport": xport, "tokens_per_s": d.get("value"),
                         "ms_per_step": d.get("ms_per_step"), "pp": d.get("config", {}).get("pp"),
                         "ep": d.get("config", {}).get("ep"), "bubble_model": d.get("config", {}).get("bubble_model")})
    return rows


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--gpus", type=int, default=0, help="measure on this many GPUs (0: simulator only)")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--steps", type=int, default=2)
    a = ap.parse_args()
    if a.gpus:
        rows = measure(a.gpus, layers=a.layers, steps=a.steps)
        if a.json:
            print(json.dumps(rows))
        else:
            print("| schedule | transport | pp x ep | tokens/s | ms/step | simulated bubble |\n|---|---|---|---|---|---|")
            for r in rows:
                tok = f"{r['tokens_per_s']:,.0f}" if r["tokens_per_s"] else "failed"
                ms = f"{r['ms_per_step']:.1f}" if r["ms_per_step"] else "-"
                print(f"| {r['schedule']} | {r['transport']} | {r['pp']}x{r['ep']} | {tok} | {ms} | {r['bubble_model']} |")
        raise SystemExit(0)
    rows = sweep()
    if a.json:
        print(json.dumps(rows))
    else:
        print("| pp | M | schedule | bubble | makespan |\n|---|---|---|---|---|")
        for r in rows:
            print(f"| {r['pp']} | {r['microbatches']} | {r['schedule']} | {r['bubble']:.3f} | {r['makespan']:.0f} |")
