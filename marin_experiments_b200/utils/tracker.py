"""Metric trackers, the per-step throughput hook, the log monitor and the step watchdog.

* ``JsonlTracker`` appends ``{"step": s, ...metrics}`` lines to ``<log_dir>/<run_id>/metrics.jsonl``
  (the role of the reference's W&B tracker with ``replicate_path``, which has no network here);
  ``NoopTracker`` drops everything (the reference's ``mode="disabled"`` on CPU).
* ``WandbTracker`` (kind ``wandb``) logs to Weights & Biases where the ``wandb`` package is installed
  (project, entity, group, tags and mode from ``WANDB_PROJECT`` / ``WANDB_ENTITY`` /
  ``WANDB_RUN_GROUP`` / ``WANDB_TAGS`` / ``WANDB_MODE``, as the reference's ``WandbConfig``) and keeps
  the JSONL copy beside it; without the package it fails at start-up with that message, never
  silently.
* ``ThroughputHook`` prints one line per step,
  ``[THRUPUT] step=N dt=1.234s tok_s=123456 mfu=0.213 bs=32``, the format the reference's sweep
  monitor parses (megagpt-speedrun/monitor.py:34-36, megagpt-speedrun/analyze_sweep.py:28);
  ``parse_thruput`` is that monitor: the median tokens/s and MFU after a warm-up.
* ``Watchdog`` is a host thread that fires when no step has finished for ``timeout_s`` seconds: it
  dumps every thread's Python stack and calls ``on_timeout`` (by default it only reports), so a hung
  collective or loader shows where it stopped.
"""

from __future__ import annotations

import faulthandler
import json
import os
import re
import statistics
import sys
import threading
import time

from .flops import training_flops_per_token


class NoopTracker:
    def log(self, metrics: dict, step: int) -> None:
        pass

    def log_summary(self, metrics: dict) -> None:
        pass

    def finish(self) -> None:
        pass


class JsonlTracker:
    def __init__(self, log_dir: str, run_id: str, config: dict | None = None):
        self.dir = os.path.join(log_dir, run_id)
        os.makedirs(self.dir, exist_ok=True)
        self.f = open(os.path.join(self.dir, "metrics.jsonl"), "a")
        if config is not None:
            with open(os.path.join(self.dir, "config.json"), "w") as f:
                json.dump(config, f, indent=1, default=str)
        self.summary: dict = {}

    def log(self, metrics: dict, step: int) -> None:
        self.f.write(json.dumps({"step": int(step), **{k: _plain(v) for k, v in metrics.items()}}) + "\n")
        self.f.flush()

    def log_summary(self, metrics: dict) -> None:
        self.summary.update({k: _plain(v) for k, v in metrics.items()})
        with open(os.path.join(self.dir, "summary.json"), "w") as f:
            json.dump(self.summary, f, indent=1)

    def finish(self) -> None:
        self.f.close()


def _plain(v):
    try:
        import torch

        if torch.is_tensor(v):
            return v.item() if v.numel() == 1 else v.tolist()
    except ImportError:
        pass
    return v


class WandbTracker:
    def __init__(self, log_dir: str, run_id: str, config: dict | None = None, *, project: str | None = None,
                 entity: str | None = None, group: str | None = None, tags: list[str] | None = None,
                 mode: str | None = None):
        try:
            import wandb
        except ImportError as e:
            raise ImportError("tracker 'wandb' needs the wandb package; use 'jsonl' without it") from e
        env = os.environ
        tags = tags if tags is not None else [t for t in env.get("WANDB_TAGS", "").split(",") if t]
        self.wandb = wandb
        self.run = wandb.init(project=project or env.get("WANDB_PROJECT", "marin_moe"),
                              entity=entity or env.get("WANDB_ENTITY"), group=group or env.get("WANDB_RUN_GROUP"),
                              name=run_id, id=run_id, resume="allow", tags=tags,
                              mode=mode or env.get("WANDB_MODE", "online"), config=config or {})
        self.jsonl = JsonlTracker(log_dir, run_id, config)

    def log(self, metrics: dict, step: int) -> None:
        plain = {k: _plain(v) for k, v in metrics.items()}
        self.run.log(plain, step=int(step))
        self.jsonl.log(plain, step)

    def log_summary(self, metrics: dict) -> None:
        plain = {k: _plain(v) for k, v in metrics.items()}
        for k, v in plain.items():
            self.run.summary[k] = v
        self.jsonl.log_summary(plain)

    def finish(self) -> None:
        self.run.finish()
        self.jsonl.finish()


def make_tracker(kind: str, log_dir: str, run_id: str, config: dict | None = None, rank: int = 0):
    if rank != 0 or kind in ("noop", "disabled", None):
        return NoopTracker()
    if kind == "jsonl":
        return JsonlTracker(log_dir, run_id, config)
    if kind == "wandb":
        return WandbTracker(log_dir, run_id, config)
    raise ValueError(f"unknown tracker {kind!r}")


class ThroughputHook:
    def __init__(self, cfg, n_gpus: int, peak_flops_per_gpu: float = 2.25e15, stream=None, every: int = 1):
        self.fpt = training_flops_per_token(cfg)
        self.n, self.peak, self.every = n_gpus, peak_flops_per_gpu, every
        self.stream = stream or sys.stdout
        self.last: dict = {}

    def __call__(self, trainer, info: dict) -> None:
        dt = info["step_duration"]
        toks = info["tokens"]
        tok_s = toks / dt if dt > 0 else float("nan")
        mfu = tok_s * self.fpt / (self.n * self.peak) if dt > 0 else float("nan")
        self.last = {"throughput/tokens_per_second": tok_s, "throughput/mfu": mfu, "throughput/step_s": dt}
        if info["step"] % self.every == 0:
            bs = info.get("batch_size", 0)
            print(f"[THRUPUT] step={info['step']} dt={dt:.3f}s tok_s={tok_s:.0f} mfu={mfu:.4f} bs={bs}",
                  file=self.stream, flush=True)


THRU = re.compile(r"\[THRUPUT\] step=(\d+) dt=([\d.]+)s tok_s=(\w+) mfu=(\w[\w.]*) bs=(\d+)")


def parse_thruput(text: str, warmup: int = 5) -> dict | None:
    """Median tokens/s and MFU of the ``[THRUPUT]`` lines at steps >= ``warmup``."""
    tps, mfus = [], []
    for m in THRU.finditer(text):
        if int(m.group(1)) >= warmup:
            if m.group(3) != "na":
                tps.append(float(m.group(3)))
            if m.group(4) != "na":
                mfus.append(float(m.group(4)))
    if not tps:
        return None
    return {"tok_s": statistics.median(tps), "mfu": statistics.median(mfus) if mfus else None, "n": len(tps)}


MAX_HIST_BUCKETS = 256


def coarsen_counts(counts, max_buckets: int = MAX_HIST_BUCKETS) -> list[float]:
    """Per-expert routing counts as a histogram of at most ``max_buckets`` buckets: adjacent experts
    are summed in equal groups (the last group zero-padded), so a log entry stays bounded for large
    expert pools (megagpt-speedrun/model.py:431-466)."""
    c = [float(x) for x in (counts.tolist() if hasattr(counts, "tolist") else counts)]
    if len(c) <= max_buckets:
        return c
    group = -(-len(c) // max_buckets)
    c += [0.0] * (-len(c) % group)
    return [sum(c[i:i + group]) for i in range(0, len(c), group)]


def router_layer_metrics(metrics: dict) -> dict:
    """Per-layer router entries for the tracker from the per-layer tensors of a step's metrics:
    ``train/router/layer_<i>/routing_entropy`` and ``train/router/layer_<i>/routing_hist``."""
    out = {}
    ent = metrics.get("routing_entropy_per_layer")
    if ent is not None:
        for i, v in enumerate(ent.float().tolist()):
            out[f"train/router/layer_{i}/routing_entropy"] = v
    cnt = metrics.get("routing_counts_per_layer")
    if cnt is not None:
        for i, row in enumerate(cnt.float().cpu()):
            out[f"train/router/layer_{i}/routing_hist"] = coarsen_counts(row)
    return out


class Watchdog:
    def __init__(self, timeout_s: float, on_timeout=None, poll_s: float | None = None, stream=None):
        self.timeout_s = timeout_s
        self.on_timeout = on_timeout
        self.poll_s = poll_s or max(0.05, min(5.0, timeout_s / 10))
        self.stream = stream or sys.stderr
        self.last = time.monotonic()
        self.fired = 0
        self._stop = threading.Event()
        self._t = None

    def start(self) -> "Watchdog":
        if self.timeout_s and self.timeout_s > 0:
            self._t = threading.Thread(target=self._run, name="step-watchdog", daemon=True)
            self._t.start()
        return self

    def kick(self, *_args) -> None:
        self.last = time.monotonic()

    __call__ = kick  # usable as a trainer hook

    def _run(self) -> None:
        while not self._stop.wait(self.poll_s):
            idle = time.monotonic() - self.last
            if idle >= self.timeout_s:
                self.fired += 1
                print(f"[watchdog] no training step finished for {idle:.1f}s; thread stacks:", file=self.stream,
                      flush=True)
                try:
                    faulthandler.dump_traceback(file=self.stream, all_threads=True)
                except (ValueError, OSError):
                    pass
                if self.on_timeout is not None:
                    self.on_timeout(idle)
                self.last = time.monotonic()

    def stop(self) -> None:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=5)
