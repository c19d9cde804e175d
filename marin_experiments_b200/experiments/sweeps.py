"""Named sweeps over the megagpt launcher's ``SP_*`` arms, run as local jobs.

The reference submits the same kind of grid to its cluster (megagpt-speedrun/iris_jobs.py:50-372:
``BASE`` environment, ``SWEEPS`` of suffix -> overrides, ``SP_TAG`` salting so the content-addressed
executor does not reuse an earlier success). Here a sweep runs on this node:

* ``plan`` expands a sweep into jobs: the arm's environment (``BASE`` + overrides + ``SP_TAG`` =
  tag-suffix, ``SP_EP`` defaulting to the GPU count), its GPU count (``_GPUS`` in an arm overrides the
  sweep's) and its command (``torch.distributed.run`` over 127.0.0.1 for more than one GPU, the plain
  launcher module otherwise). ``_BATCH_PER_GPU`` in an arm sets ``SP_BATCH`` to that times the GPUs
  (weak-scaling ladders).
* ``run`` executes the jobs one after another, each in its own process group under a time limit
  (on expiry that group alone is killed), writes ``<log_dir>/<name>.log`` (its output) and
  ``<name>.cmd`` (its environment and command) per arm and returns the logs; ``main`` then prints
  ``utils.analysis.sweep_table`` over them (median ``[THRUPUT]`` after the warm-up steps, failure
  kind per run).
* ``submit`` instead sends every arm as a job to the client that ``MXK_CLUSTER`` names (``cluster``:
  this node's GPU-slot scheduler, so arms that fit run side by side, or another host over SSH); with
  ``--wait`` it collects each job's log into ``<log_dir>`` and prints the same table.

Usage: ``python -m marin_experiments_b200.experiments.sweeps <sweep> [--only a,b] [--tag T]
[--gpus N] [--log-dir D] [--timeout S] [--dry-run] [--submit [--wait]]``.
"""

from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
from dataclasses import dataclass, field

LAUNCHER = "marin_experiments_b200.experiments.megagpt"

# Synthetic data, one [THRUPUT] line per step, the megagpt geometry from the AdamH heuristic.
BASE = {
    "SP_DATA": "synthetic", "SP_SYNTH_DATA": "1", "SP_LOG_EVERY": "1", "SP_STEPS": "30",
    "SP_TOKENS": "2000000000", "SP_HIDDEN": "1536", "SP_EXPERTS": "64", "SP_TOPK": "4", "SP_SEQ": "2048",
    "SP_BATCH": "32", "SP_REMAT": "none", "SP_ATTN": "sm100_flash",
}

# real data at constant LR (the stable phase of a warmup-stable-decay schedule)
_REAL = {"SP_SYNTH_DATA": "0", "SP_DATA": "datakit", "SP_SCHEDULE": "constant", "SP_WARMUP": "0.02",
         "SP_TOKENS": "5400000000"}
NEEDS_INIT = ("cool", "eval")

SWEEPS: dict[str, dict[str, dict[str, str]]] = {
    # the expert ladder at the headline geometry
    "anchor": {
        "e64k4": {},
        "e64k8": {"SP_TOPK": "8"},
        "e128k8": {"SP_EXPERTS": "128", "SP_TOPK": "8"},
        "e256k8": {"SP_EXPERTS": "256", "SP_TOPK": "8", "SP_BATCH": "16"},
    },
    # expert parallelism vs replicated experts (data parallel) on the same GPUs
    "dp": {
        "ep": {},
        "dp": {"SP_EP": "1"},
    },
    # throughput levers one at a time
    "lever": {
        "base": {},
        "embed512": {"SP_EMBED": "512"},
        "local_attn": {"SP_GLOBAL_EVERY": "4", "SP_LOCAL_WINDOW": "1024"},
        "remat_moe": {"SP_REMAT": "save_moe"},
        "remat_all": {"SP_REMAT": "recompute_all"},
        "fast_qb": {"SP_FAST_QB": "1"},
    },
    # largest batch that fits: per-GPU sequences 8 .. 64
    "mem": {f"b{b}": {"_BATCH_PER_GPU": str(b)} for b in (8, 16, 32, 64)},
    # short runs for a profile capture
    "prof": {"prof": {"SP_STEPS": "12"}},
    # weak scaling at 32 sequences per GPU
    "weak": {f"g{g}": {"_GPUS": str(g), "_BATCH_PER_GPU": "32"} for g in (1, 2, 4, 8)},
    # loss against wall-clock on real data, constant LR: more experts vs wider experts vs the base; each
    # arm's step count sized to end near the same time (megagpt-speedrun/iris_jobs.py "lossab")
    "lossab": {
        "a_thin": {"SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "save_moe", **_REAL, "SP_STEPS": "23000"},
        "b_bigE": {"SP_EXPERTS": "256", "SP_TOPK": "8", "SP_BATCH": "8", "SP_REMAT": "save_moe", **_REAL,
                   "SP_STEPS": "48000"},
        "c_chonky": {"SP_TOPK": "8", "SP_BATCH": "16", "SP_INTERMEDIATE": "1536", "SP_REMAT": "recompute_all",
                     **_REAL, "SP_STEPS": "13000"},
    },
    # wider experts at batches that fit
    "best": {
        "chonky2x_b16": {"SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "recompute_all", "SP_INTERMEDIATE": "1536"},
        "chonky4x_b8": {"SP_TOPK": "8", "SP_BATCH": "8", "SP_REMAT": "recompute_all", "SP_INTERMEDIATE": "3072"},
    },
    # model-size ladder at b16: more experts, wider experts, wider model (the reference's scale rounds)
    "scale": {
        "e128k8": {"SP_EXPERTS": "128", "SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "save_moe"},
        "e256k8": {"SP_EXPERTS": "256", "SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "save_moe"},
        "e256k16": {"SP_EXPERTS": "256", "SP_TOPK": "16", "SP_BATCH": "16", "SP_REMAT": "save_moe"},
        "e128i1536": {"SP_EXPERTS": "128", "SP_TOPK": "8", "SP_BATCH": "16", "SP_INTERMEDIATE": "1536",
                      "SP_REMAT": "recompute_all"},
        "d2048e128": {"SP_HIDDEN": "2048", "SP_EXPERTS": "128", "SP_TOPK": "8", "SP_BATCH": "16",
                      "SP_REMAT": "save_moe"},
    },
    "scale2": {
        "e192k8": {"SP_EXPERTS": "192", "SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "save_moe"},
        "e64i1536": {"SP_TOPK": "8", "SP_BATCH": "16", "SP_INTERMEDIATE": "1536", "SP_REMAT": "recompute_all"},
        "e128i1024": {"SP_EXPERTS": "128", "SP_TOPK": "8", "SP_BATCH": "16", "SP_INTERMEDIATE": "1024",
                      "SP_REMAT": "recompute_all"},
        "e256k8b8": {"SP_EXPERTS": "256", "SP_TOPK": "8", "SP_BATCH": "8", "SP_REMAT": "save_moe"},
        "d2048e64": {"SP_HIDDEN": "2048", "SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "save_moe"},
    },
    "scale3": {f"e{e}k8": {"SP_EXPERTS": str(e), "SP_TOPK": "8", "SP_BATCH": "16", "SP_REMAT": "save_moe"}
               for e in (144, 160, 176)},
    # the production pretraining arm: E128 / K8 at sequence 4096 on real data, constant LR
    "run2": {"e128k8": {"SP_EXPERTS": "128", "SP_TOPK": "8", "SP_BATCH": "16", "SP_SEQ": "4096",
                        "SP_REMAT": "save_moe", **_REAL, "SP_MIN_LR": "0", "SP_TOKENS": "13500000000",
                        "SP_STEPS": "205000"}},
    # SFT cooldown of a run2 checkpoint (weights only; needs --init-from): chat data, linear decay to 0
    "cool": {"sft": {"SP_EXPERTS": "128", "SP_TOPK": "8", "SP_BATCH": "16", "SP_SEQ": "4096", "SP_REMAT": "save_moe",
                     "SP_SYNTH_DATA": "0", "SP_DATA": "sft", "SP_SCHEDULE": "linear", "SP_MIN_LR": "0",
                     "SP_WARMUP": "0.02", "SP_TOKENS": "13500000000", "SP_STEPS": "20000"}},
    # held-out evaluation of a checkpoint, no training (needs --init-from)
    "eval": {"spr1": {"SP_TOPK": "8", "SP_BATCH": "16", "SP_SEQ": "4096", "SP_REMAT": "save_moe",
                      "SP_SYNTH_DATA": "0", "SP_DATA": "datakit_eval", "SP_STEPS": "1000", "SP_EVAL": "1",
                      "SP_EVAL_ONLY": "1", "SP_EVAL_BS": "16"}},
    # adaptive sparsity and the k curriculum
    "sparsity": {
        "fixed": {},
        "adapt": {"SPARSITY_MODE": "adaptive", "SP_MIN_K": "1", "SP_COEF": "0.01"},
        "curric": {"SP_CURRICULUM": "2:0.5,4:1.0"},
    },
    # the pipeline-parallel entry points
    "pp": {
        "pp_sync": {"SP_PP_MODE": "sync"},
        "pp_async": {"SP_PP_MODE": "async"},
    },
}


@dataclass
class Job:
    name: str
    gpus: int
    env: dict[str, str] = field(default_factory=dict)
    argv: list[str] = field(default_factory=list)


def command(gpus: int, port: int, module: str = LAUNCHER) -> list[str]:
    if gpus <= 1:
        return [sys.executable, "-m", module]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr", "127.0.0.1", f"--master-port={port}", "-m", module]


def plan(sweep: str, *, gpus: int = 8, tag: str = "sw", only: list[str] | None = None, port: int = 29611,
         module: str = LAUNCHER, sweeps: dict | None = None) -> list[Job]:
    grid = (sweeps or SWEEPS)[sweep]
    jobs = []
    for i, (suffix, over) in enumerate(grid.items()):
        if only and suffix not in only:
            continue
        over = dict(over)
        g = int(over.pop("_GPUS", gpus))
        env = dict(BASE)
        env["SP_EP"] = str(g)
        per_gpu = over.pop("_BATCH_PER_GPU", None)
        env.update(over)
        if per_gpu is not None:
            env["SP_BATCH"] = str(int(per_gpu) * g)
        env["SP_TAG"] = f"{tag}-{suffix}"
        jobs.append(Job(f"{tag}-{suffix}", g, env, command(g, port + i, module)))
    if only:
        missing = set(only) - set(grid)
        if missing:
            raise KeyError(f"sweep {sweep!r} has no arm(s) {sorted(missing)}")
    return jobs


def describe(job: Job) -> str:
    env = " ".join(f"{k}={v}" for k, v in sorted(job.env.items()))
    return f"[{job.name}] gpus={job.gpus}  {env}  {' '.join(job.argv)}"


def run(jobs: list[Job], log_dir: str, *, timeout_s: float = 3600.0, dry_run: bool = False) -> list[str]:
    """Run each job to completion (or its time limit); returns the log paths in order."""
    os.makedirs(log_dir, exist_ok=True)
    logs = []
    for job in jobs:
        path = os.path.join(log_dir, f"{job.name}.log")
        logs.append(path)
        if dry_run:
            print(describe(job), flush=True)
            continue
        with open(os.path.join(log_dir, f"{job.name}.cmd"), "w") as f:
            f.write(describe(job) + "\n")
        with open(path, "w") as f:
            p = subprocess.Popen(job.argv, env={**os.environ, **job.env}, stdout=f, stderr=subprocess.STDOUT,
                                 start_new_session=True)
            try:
                rc = p.wait(timeout=timeout_s)
            except subprocess.TimeoutExpired:
                os.killpg(p.pid, signal.SIGKILL)  # this job's own process group only
                p.wait()
                rc = "timeout"
                f.write(f"\n[sweep] killed after {timeout_s:.0f}s\n")
            f.write(f"\n[sweep] exit {rc}\n")
        print(f"[sweep] {job.name}: exit {rc} -> {path}", flush=True)
    return logs


def submit(jobs: list[Job], client, *, timeout_s: float = 3600.0, retries: int = 0) -> list:
    """Send each arm to ``client`` (``cluster.LocalClient`` / ``SSHClient``); returns the job handles.
    The client starts a multi-GPU Python job under ``torch.distributed.run`` itself, so an arm's own
    torchrun prefix is dropped."""
    from .. import cluster as C

    handles = []
    for job in jobs:
        argv = list(job.argv)
        if argv[1:3] == ["-m", "torch.distributed.run"]:
            argv = [argv[0]] + argv[argv.index("-m", 3):]
        req = C.JobRequest(job.name, C.Entrypoint.from_command(*argv), C.ResourceConfig(gpus=job.gpus),
                           dict(job.env), retries, timeout_s)
        handles.append(client.submit(req))
    return handles


def collect(handles: list, names: list[str], log_dir: str) -> list[str]:
    """Wait for submitted arms and copy each job's log to ``<log_dir>/<name>.log``."""
    import shutil

    os.makedirs(log_dir, exist_ok=True)
    logs = []
    for h, name in zip(handles, names):
        state = h.wait(raise_on_failure=False)
        path = os.path.join(log_dir, f"{name}.log")
        if os.path.exists(h.log_path()):
            shutil.copyfile(h.log_path(), path)
        with open(path, "a") as f:
            f.write(f"\n[sweep] job {h.job_id} {state} exit {h.exit_code}\n")
        print(f"[sweep] {name}: {state} -> {path}", flush=True)
        logs.append(path)
    return logs


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m marin_experiments_b200.experiments.sweeps")
    ap.add_argument("sweep", choices=sorted(SWEEPS))
    ap.add_argument("--only", default=None, help="comma-separated arm suffixes")
    ap.add_argument("--tag", default="sw")
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--log-dir", default="sweep_logs")
    ap.add_argument("--timeout", type=float, default=3600.0)
    ap.add_argument("--warmup", type=int, default=8, help="steps excluded from the tokens/s median")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--init-from", default=None, help="checkpoint for weights-only init (SP_INIT_FROM)")
    ap.add_argument("--submit", action="store_true", help="send the arms to a job scheduler instead of running them")
    ap.add_argument("--wait", action="store_true", help="with --submit: wait and analyse the logs")
    a = ap.parse_args(argv)
    if a.sweep in NEEDS_INIT and not a.init_from:
        raise SystemExit(f"sweep {a.sweep} needs --init-from <checkpoint directory>")
    jobs = plan(a.sweep, gpus=a.gpus, tag=a.tag, only=a.only.split(",") if a.only else None)
    if a.init_from:
        for j in jobs:
            j.env["SP_INIT_FROM"] = a.init_from
    if a.submit and not a.dry_run:
        from ..cluster import current_client

        handles = submit(jobs, current_client(), timeout_s=a.timeout)
        for h, job in zip(handles, jobs):
            print(f"[sweep] submitted {job.name} -> {h.job_id}", flush=True)
        if not a.wait:
            return 0
        logs = collect(handles, [j.name for j in jobs], a.log_dir)
    else:
        logs = run(jobs, a.log_dir, timeout_s=a.timeout, dry_run=a.dry_run)
    if not a.dry_run:
        from ..utils.analysis import analyze_logs, sweep_table

        print(sweep_table(analyze_logs(logs, warmup=a.warmup)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
