"""Run analysis: sweep logs, tracker histories and device-time breakdowns of a profiled step.

The reference does this with separate scripts against its cluster and W&B
(megagpt-speedrun/analyze_sweep.py:33-99, megagpt-speedrun/collect_results.py:28-106,
megagpt-speedrun/iso_step.py:33-95, megagpt-speedrun/analyze_profile.py:63-157). Here the inputs are
local files written by this framework:

* **sweep logs** (``analyze_logs``): one stdout log per run (the CLI's ``--watch N`` re-reads them
  every N seconds while runs are going, with glob patterns picking up new logs). The ``[arm]`` line (printed by the
  megagpt launcher) gives the geometry, the ``[THRUPUT]`` lines give per-step tokens/s and MFU (the
  median over steps >= warm-up is the run's number), and the first failure signature (out of
  memory, NCCL error, watchdog, NaN stop, segfault, CUDA fault) marks runs that died.
* **tracker histories** (``collect_results``, ``iso_step``): ``metrics.jsonl`` / ``summary.json``
  under ``<log_dir>/<run_id>/`` from ``utils.tracker.JsonlTracker``. ``iso_step`` reads each run's
  value at a common step (the last logged row at or before it), so runs that stopped early are
  compared at the same point rather than at their final values.
* **profiles** (``profile_breakdown``): a Chrome trace exported by ``torch.profiler`` (``.json`` or
  ``.json.gz``). Device events (kernels, memcpy, memset) are summed by name and rolled into this
  framework's kernel families, so the table says where a step's device time goes. ``profile_call``
  records such a trace around a callable.
"""

from __future__ import annotations

import argparse
import gzip
import json
import os
import re
import statistics
from collections import defaultdict
from dataclasses import dataclass, field

from .tracker import THRU

ARM = re.compile(r"\[arm\]\s+(?P<run>\S+).*?D=(?P<D>\d+).*?seq=(?P<seq>\d+) E=(?P<E>\d+) k=(?P<k>\d+)"
                 r".*?batch=(?P<batch>\d+).*?budget=(?P<budget>[\d.eE+-]+)")
FAILURES = [
    ("oom", re.compile(r"out of memory|OutOfMemoryError|RESOURCE_EXHAUSTED", re.I)),
    ("nccl", re.compile(r"NCCL (error|WARN.*(timeout|abort))|ProcessGroupNCCL.*(timeout|Watchdog caught)", re.I)),
    ("watchdog", re.compile(r"\[watchdog\]")),
    ("nan", re.compile(r"loss is (nan|-?inf)\b|FloatingPointError", re.I)),
    ("cuda_fault", re.compile(r"illegal (memory access|instruction)|misaligned address|device-side assert|"
                              r"unspecified launch failure", re.I)),
    ("segfault", re.compile(r"Segmentation fault|Fatal Python error|SIGSEGV")),
    ("kernel_timeout", re.compile(r"KernelTimeoutError|kernel wait timed out")),
]


@dataclass
class LogRun:
    path: str
    arm: dict = field(default_factory=dict)
    tok_s: float | None = None
    mfu: float | None = None
    n_steps: int = 0
    last_step: int | None = None
    failure: str = ""


def classify_failure(text: str) -> str:
    """First failure kind whose signature appears in ``text`` (``""`` if none)."""
    best = None
    for kind, pat in FAILURES:
        m = pat.search(text)
        if m and (best is None or m.start() < best[1]):
            best = (kind, m.start())
    return best[0] if best else ""


def analyze_log(text: str, warmup: int = 8, path: str = "") -> LogRun:
    run = LogRun(path=path)
    m = ARM.search(text)
    if m:
        g = m.groupdict()
        run.arm = {"run": g["run"], **{k: int(g[k]) for k in ("D", "seq", "E", "k", "batch")},
                   "budget": float(g["budget"])}
    tps, mfus, steps = [], [], []
    for t in THRU.finditer(text):
        step = int(t.group(1))
        steps.append(step)
        if step < warmup:
            continue
        if t.group(3) != "na":
            tps.append(float(t.group(3)))
        if t.group(4) != "na":
            mfus.append(float(t.group(4)))
    run.n_steps = len(tps)
    run.last_step = max(steps) if steps else None
    run.tok_s = statistics.median(tps) if tps else None
    run.mfu = statistics.median(mfus) if mfus else None
    run.failure = classify_failure(text)
    return run


def analyze_logs(paths: list[str], warmup: int = 8) -> list[LogRun]:
    out = []
    for p in paths:
        with open(p, errors="replace") as f:
            out.append(analyze_log(f.read(), warmup=warmup, path=p))
    return out


def sweep_table(runs: list[LogRun]) -> str:
    """Markdown table, fastest first; failed runs and runs without steady-state steps last."""
    rows = ["| run | D | E | k | batch | tok/s | MFU | steps | last step | failure |",
            "|---|---|---|---|---|---|---|---|---|---|"]
    for r in sorted(runs, key=lambda r: (bool(r.failure) or r.tok_s is None, -(r.tok_s or 0.0))):
        a = r.arm
        name = a.get("run") or os.path.basename(os.path.dirname(r.path) or r.path) or r.path
        tok = f"{r.tok_s:,.0f}" if r.tok_s is not None else "-"
        mfu = f"{r.mfu:.3f}" if r.mfu is not None else "-"
        rows.append(f"| {name} | {a.get('D', '-')} | {a.get('E', '-')} | {a.get('k', '-')} | "
                    f"{a.get('batch', '-')} | {tok} | {mfu} | {r.n_steps} | "
                    f"{r.last_step if r.last_step is not None else '-'} | {r.failure} |")
    return "\n".join(rows)


# ------------------------------------------------------------------------------------------ tracker
def load_history(run_dir: str) -> list[dict]:
    """Rows of ``metrics.jsonl`` sorted by step (a torn last line from a killed run is skipped)."""
    rows = []
    path = os.path.join(run_dir, "metrics.jsonl")
    if not os.path.exists(path):
        return rows
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                rows.append(json.loads(line))
            except json.JSONDecodeError:
                continue
    rows.sort(key=lambda r: r.get("step", 0))
    return rows


def value_at_step(history: list[dict], step: int, key: str) -> tuple[float | None, int | None]:
    """``key`` at the last row with step <= ``step`` that has it; the first such row if none is that
    early. Returns (value, the step it came from)."""
    have = [r for r in history if r.get(key) is not None]
    if not have:
        return None, None
    le = [r for r in have if r["step"] <= step]
    row = le[-1] if le else have[0]
    return float(row[key]), int(row["step"])


def run_dirs(log_dir: str, pattern: str | None = None) -> list[str]:
    """Run directories under ``log_dir`` (those holding ``metrics.jsonl``), optionally filtered by a
    regular expression on the run id."""
    rx = re.compile(pattern) if pattern else None
    out = []
    for name in sorted(os.listdir(log_dir)):
        d = os.path.join(log_dir, name)
        if os.path.exists(os.path.join(d, "metrics.jsonl")) and (rx is None or rx.search(name)):
            out.append(d)
    return out


def collect_results(dirs: list[str], keys: list[str]) -> list[dict]:
    """Final values per run: ``summary.json`` where written, else the last logged value."""
    out = []
    for d in dirs:
        hist = load_history(d)
        summary = {}
        sp = os.path.join(d, "summary.json")
        if os.path.exists(sp):
            with open(sp) as f:
                summary = json.load(f)
        row = {"run": os.path.basename(d), "max_step": hist[-1]["step"] if hist else None}
        for k in keys:
            if k in summary:
                row[k] = summary[k]
            else:
                v, _ = value_at_step(hist, 1 << 62, k)
                row[k] = v
        out.append(row)
    return out


def iso_step(dirs: list[str], step: int, keys: list[str]) -> list[dict]:
    """Each run's ``keys`` at a common ``step`` (plus the step each value came from and the run's
    last logged step)."""
    out = []
    for d in dirs:
        hist = load_history(d)
        row = {"run": os.path.basename(d), "max_step": hist[-1]["step"] if hist else None}
        for k in keys:
            v, s = value_at_step(hist, step, k)
            row[k], row[f"{k}@step"] = v, s
        out.append(row)
    return out


def smooth(values, window: int):
    """Centred rolling mean that averages only the points that exist near the ends (no zero padding,
    which would pull the final values -- the plateau this analysis reads -- towards zero)."""
    import numpy as np

    v = np.asarray(values, dtype=np.float64)
    if window <= 1 or len(v) == 0:
        return v
    c = np.concatenate([[0.0], np.cumsum(v)])
    h = window // 2
    lo = np.clip(np.arange(len(v)) - h, 0, len(v))
    hi = np.clip(np.arange(len(v)) + window - h, 0, len(v))
    return (c[hi] - c[lo]) / (hi - lo)


def isoloss(histories: dict[str, list[tuple[int, float]]], sync: str, *, tail_frac: float = 0.1,
            window: int = 25) -> list[dict]:
    """Token overhead of delayed / pipelined runs against a synchronous reference
    (delayed-gradient-pp/analyze_isoloss.py). Per run, from its ``(step, loss)`` history:

    * ``plateau``: mean of the raw losses over the last ``tail_frac`` of the steps;
    * ``gap``: plateau minus the reference's plateau;
    * ``slope_per_1k``: least-squares slope over that tail, per 1000 steps (still negative: the run
      is still descending -- a token tax, not a floor);
    * ``overhead``: the first step at which the run's smoothed loss reaches its own plateau, over the
      first step at which the reference's smoothed loss reaches that same value (tokens scale with
      steps at a fixed batch); ``None`` when the reference never gets there."""
    import numpy as np

    def stats(h):
        h = sorted(h)
        steps = np.array([s for s, _ in h], dtype=np.float64)
        loss = np.array([v for _, v in h], dtype=np.float64)
        n = max(2, int(round(len(h) * tail_frac)))
        ts, tl = steps[-n:], loss[-n:]
        slope = float(np.polyfit(ts, tl, 1)[0]) * 1000 if len(ts) >= 2 and ts[-1] > ts[0] else 0.0
        return steps, loss, smooth(loss, window), float(tl.mean()), slope

    if sync not in histories:
        raise KeyError(f"reference run {sync!r} not among {sorted(histories)}")
    s_steps, _, s_sm, s_plat, _ = stats(histories[sync])
    out = []
    for name, h in histories.items():
        steps, _, sm, plat, slope = stats(h)
        reach = np.nonzero(sm <= plat)[0]
        own = float(steps[reach[0]]) if len(reach) else float(steps[-1])
        ref = np.nonzero(s_sm <= plat)[0]
        overhead = own / float(s_steps[ref[0]]) if len(ref) and s_steps[ref[0]] > 0 else None
        out.append({"run": name, "plateau": plat, "gap": plat - s_plat, "slope_per_1k": slope,
                    "overhead": overhead, "steps": int(steps[-1])})
    return out


def rows_table(rows: list[dict], keys: list[str]) -> str:
    head = ["run", "max_step"] + keys
    lines = ["| " + " | ".join(head) + " |", "|" + "---|" * len(head)]
    for r in rows:
        cells = [str(r["run"]), str(r["max_step"])]
        for k in keys:
            v = r.get(k)
            cells.append(f"{v:.4f}" if isinstance(v, float) else ("-" if v is None else str(v)))
        lines.append("| " + " | ".join(cells) + " |")
    return "\n".join(lines)


# ----------------------------------------------------------------------------------------- profiles
# Kernel families of this framework: regular expressions tried in order on the lower-cased device
# event name (the first match wins).
CATEGORIES = [
    (r"nccl", "collective (NCCL)"),
    (r"\bep_", "EP exchange (NVLink peer kernels)"),
    (r"fa_bwd|flash_bwd|dq_convert", "attention backward"),
    (r"fa_fwd|flash_fwd|decode_attn|decode_combine", "attention forward"),
    (r"gemm_sm100", "GEMM (tcgen05)"),
    (r"gemm|cutlass|cublas|\bsm\d+_xmma", "GEMM (library)"),
    (r"router|qb_beta", "router / QB"),
    (r"plan_|noalloc_|permute|combine|gather_k|ep_push|ep_wait|ep_signal|ep_dispatch|ep_unpermute", "MoE dispatch / combine"),
    (r"\bce_", "cross-entropy"),
    (r"adamh|moments_|sqnorm|\bema_|optim", "optimizer"),
    (r"rmsnorm|qk_norm|head_norm|xsa_gate|gate_mul", "norms / rope / gates"),
    (r"swiglu|\bact_", "activations"),
    (r"embed|ngram|kv_append", "embedding / cache"),
    (r"memcpy|memset|copy|cast_bf16", "copy / memset"),
    (r"elementwise|reduce_kernel|vectorized|unrolled", "torch elementwise"),
]
_CAT_RX = [(re.compile(p), c) for p, c in CATEGORIES]
DEVICE_CATS = {"kernel", "gpu_memcpy", "gpu_memset"}


def categorize(name: str) -> str:
    n = name.lower()
    for rx, cat in _CAT_RX:
        if rx.search(n):
            return cat
    return "other"


def load_trace(path: str) -> list[dict]:
    opener = gzip.open if path.endswith(".gz") else open
    with opener(path, "rt") as f:
        data = json.load(f)
    return data["traceEvents"] if isinstance(data, dict) else data


def profile_breakdown(events: list[dict], steps: int = 1, top: int = 15) -> dict:
    """Device time by kernel family and the ``top`` kernels, in ms per step, from Chrome-trace events.
    Durations are in microseconds in the trace format."""
    by_name: dict[str, float] = defaultdict(float)
    count: dict[str, int] = defaultdict(int)
    for e in events:
        if e.get("ph") != "X" or e.get("cat") not in DEVICE_CATS:
            continue
        by_name[e.get("name", "?")] += float(e.get("dur", 0.0))
        count[e.get("name", "?")] += 1
    by_cat: dict[str, float] = defaultdict(float)
    for n, us in by_name.items():
        by_cat[categorize(n)] += us
    total = sum(by_cat.values())
    per = max(steps, 1) * 1e3
    cats = sorted(((c, us / per, us / total if total else 0.0) for c, us in by_cat.items()), key=lambda x: -x[1])
    kernels = sorted(((n, us / per, count[n] / max(steps, 1), categorize(n)) for n, us in by_name.items()),
                     key=lambda x: -x[1])[:top]
    return {"total_ms_per_step": total / per, "categories": cats, "top_kernels": kernels,
            "launches_per_step": sum(count.values()) / max(steps, 1)}


def breakdown_table(b: dict) -> str:
    lines = [f"device time {b['total_ms_per_step']:.2f} ms/step, {b['launches_per_step']:.0f} launches/step", "",
             "| family | ms/step | share |", "|---|---|---|"]
    lines += [f"| {c} | {ms:.2f} | {sh:.1%} |" for c, ms, sh in b["categories"]]
    lines += ["", "| kernel | ms/step | launches/step | family |", "|---|---|---|---|"]
    lines += [f"| {n[:90]} | {ms:.3f} | {cnt:g} | {c} |" for n, ms, cnt, c in b["top_kernels"]]
    return "\n".join(lines)


def profile_call(fn, steps: int = 1, trace_path: str | None = None, top: int = 40) -> dict:
    """Run ``fn()`` ``steps`` times under ``torch.profiler`` (CPU + CUDA activity) and return
    ``profile_breakdown`` of the device events. Numbers taken this way are for shares only: the
    profiler adds overhead, so step times come from the un-profiled benchmark."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    path = trace_path or os.path.join(os.getcwd(), "step_trace.json")
    with profile(activities=acts) as prof:
        for _ in range(steps):
            fn()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    prof.export_chrome_trace(path)
    return profile_breakdown(load_trace(path), steps=steps, top=top)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m marin_experiments_b200.utils.analysis")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("sweep", help="tokens/s table from run stdout logs")
    s.add_argument("logs", nargs="+")
    s.add_argument("--warmup", type=int, default=8)
    s.add_argument("--watch", type=float, default=0.0, help="re-read the logs every N seconds (0: once)")
    s.add_argument("--rounds", type=int, default=0, help="with --watch: stop after this many tables (0: never)")
    c = sub.add_parser("results", help="final tracker values per run")
    c.add_argument("log_dir")
    c.add_argument("--match", default=None)
    c.add_argument("--keys", default="train/loss")
    i = sub.add_parser("iso-step", help="tracker values at a common step")
    i.add_argument("log_dir")
    i.add_argument("--step", type=int, required=True)
    i.add_argument("--match", default=None)
    i.add_argument("--keys", default="train/loss")
    q = sub.add_parser("isoloss", help="token overhead of runs against a synchronous reference run")
    q.add_argument("log_dir")
    q.add_argument("--sync", required=True, help="run id of the synchronous reference")
    q.add_argument("--match", default=None)
    q.add_argument("--key", default="train/loss")
    q.add_argument("--tail", type=float, default=0.1)
    q.add_argument("--window", type=int, default=25)
    p = sub.add_parser("profile", help="device-time breakdown of a torch.profiler Chrome trace")
    p.add_argument("trace")
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--top", type=int, default=15)
    a = ap.parse_args(argv)
    if a.cmd == "sweep":
        import glob
        import time

        n = 0
        while True:
            paths = sorted({p for pat in a.logs for p in (glob.glob(pat) or [pat]) if os.path.exists(p)})
            print(sweep_table(analyze_logs(paths, a.warmup)), flush=True)
            n += 1
            if a.watch <= 0 or (a.rounds and n >= a.rounds):
                break
            time.sleep(a.watch)
    elif a.cmd == "isoloss":
        hist = {os.path.basename(d): [(int(r["step"]), float(r[a.key])) for r in load_history(d)
                                      if r.get(a.key) is not None] for d in run_dirs(a.log_dir, a.match)}
        rows = isoloss({k: v for k, v in hist.items() if v}, a.sync, tail_frac=a.tail, window=a.window)
        keys = ["plateau", "gap", "slope_per_1k", "overhead"]
        print(rows_table([{**r, "max_step": r["steps"]} for r in rows], keys))
    elif a.cmd in ("results", "iso-step"):
        keys = a.keys.split(",")
        dirs = run_dirs(a.log_dir, a.match)
        rows = collect_results(dirs, keys) if a.cmd == "results" else iso_step(dirs, a.step, keys)
        print(rows_table(rows, keys if a.cmd == "results" else sum(([k, f"{k}@step"] for k in keys), [])))
    else:
        print(breakdown_table(profile_breakdown(load_trace(a.trace), a.steps, a.top)))


if __name__ == "__main__":
    main()
