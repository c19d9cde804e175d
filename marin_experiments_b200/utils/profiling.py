"""Step profiling, NVTX ranges and watch statistics.

* ``ProfilerHook``: records a ``torch.profiler`` trace (CPU + CUDA activity) over training steps
  ``[start_step, start_step + num_steps)`` and writes ``<out_dir>/trace.json`` plus the device-time
  breakdown by kernel family (``utils.analysis``) as ``<out_dir>/breakdown.md`` (the reference's
  ``ProfilerConfig(enabled, start_step, num_steps)`` hook, megagpt-speedrun/train.py:645-677, with
  the category rollup of megagpt-speedrun/analyze_profile.py).
* ``nvtx_range``: a named range around a host phase (forward / backward per microbatch, gradient
  sync, optimizer) when ``MXK_NVTX=1``, so a profiler's timeline and ``ncu --nvtx-include`` can select
  phases (the role of the reference's ``TraceAnnotation`` marks, megagpt-speedrun/train.py:720,738);
  a no-op otherwise.
* ``watch_stats``: gradient and parameter norms by parameter kind (and optionally per parameter),
  plus a coarse histogram of the gradient values (megagpt-speedrun/train.py:484-497). Expert-sharded
  parameters' squared sums are added over the expert-parallel group, so every rank reports the
  norms of the whole model.
"""

from __future__ import annotations

import contextlib
import math
import os

import torch


@contextlib.contextmanager
def nvtx_range(name: str):
    if os.environ.get("MXK_NVTX") == "1" and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class ProfilerHook:
    """Pre-step hook (``before_step``) starts the profiler when the trainer reaches ``start_step``;
    post-step hook (``__call__``) stops it after ``num_steps`` steps and writes the trace and the
    breakdown (rank 0 writes; every rank records so that all ranks run the same steps)."""

    def __init__(self, out_dir: str, start_step: int = 5, num_steps: int = 5, rank: int = 0):
        self.out_dir, self.start, self.num, self.rank = out_dir, start_step, max(1, num_steps), rank
        self.prof = None
        self.done = False
        self.breakdown: dict | None = None

    def before_step(self, trainer) -> None:
        if self.done or self.prof is not None or trainer.step != self.start:
            return
        from torch.profiler import ProfilerActivity, profile

        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
        self.prof = profile(activities=acts)
        self.prof.__enter__()

    def __call__(self, trainer, info: dict) -> None:
        if self.prof is None or info["step"] < self.start + self.num:
            return
        from .analysis import breakdown_table, load_trace, profile_breakdown

        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.prof.__exit__(None, None, None)
        if self.rank == 0:
            os.makedirs(self.out_dir, exist_ok=True)
            path = os.path.join(self.out_dir, "trace.json")
            self.prof.export_chrome_trace(path)
            self.breakdown = profile_breakdown(load_trace(path), steps=self.num)
            with open(os.path.join(self.out_dir, "breakdown.md"), "w") as f:
                f.write(f"steps {self.start}..{self.start + self.num - 1}\n\n" + breakdown_table(self.breakdown) + "\n")
        self.prof = None
        self.done = True


def _kind(name: str) -> str:
    """Parameter kind: the owning module's name without layer indices + the leaf
    (``blocks.3.mlp.w_gate_up`` -> ``mlp.w_gate_up``)."""
    parts = [p for p in name.split(".") if not p.isdigit()]
    return ".".join(parts[-2:]) if len(parts) >= 2 else parts[0]


def watch_stats(store, *, per_param: bool = False, hist_bins: int = 0, hist_range: float = 1e-2,
                ep_group=None) -> dict[str, float]:
    """Norms of the gradients (as accumulated for the optimizer) and parameters (fp32 master) of
    ``store``: ``watch/grad_norm/<kind>``, ``watch/param_norm/<kind>`` and the totals; with
    ``per_param`` also per parameter name; with ``hist_bins`` a histogram of the gradient values over
    ``[-hist_range, hist_range]`` as ``watch/grad_hist`` (a list of counts, values outside clamped
    into the end bins). One host synchronisation."""
    kinds: dict[str, int] = {}
    names = []
    rows = []
    shard = []
    for info in store.infos:
        g = store.grad[info.offset: info.offset + info.numel]
        p = store.master[info.offset: info.offset + info.numel]
        rows.append(torch.stack([g.float().square().sum(), p.float().square().sum()]))
        names.append(info.name)
        shard.append(getattr(info, "sharded_over", None) == "expert")
        kinds.setdefault(_kind(info.name), len(kinds))
    if not rows:
        return {}
    sq = torch.stack(rows)  # [n_params, 2]
    if ep_group is not None and any(shard):
        mask = torch.tensor(shard, device=sq.device)
        part = sq * mask[:, None]
        torch.distributed.all_reduce(part, group=ep_group)
        sq = torch.where(mask[:, None], part, sq)
    hist = None
    if hist_bins > 0:
        hist = torch.histc(store.grad.float().clamp(-hist_range, hist_range), bins=hist_bins, min=-hist_range,
                           max=hist_range)
    vals = sq.tolist()
    out: dict[str, float] = {}
    by_kind: dict[str, list[float]] = {}
    for name, (gs, ps) in zip(names, vals):
        k = _kind(name)
        acc = by_kind.setdefault(k, [0.0, 0.0])
        acc[0] += gs
        acc[1] += ps
        if per_param:
            out[f"watch/grad_norm/{name}"] = math.sqrt(gs)
            out[f"watch/param_norm/{name}"] = math.sqrt(ps)
    for k, (gs, ps) in by_kind.items():
        out[f"watch/grad_norm/{k}"] = math.sqrt(gs)
        out[f"watch/param_norm/{k}"] = math.sqrt(ps)
    out["watch/grad_norm/total"] = math.sqrt(sum(v[0] for v in by_kind.values()))
    out["watch/param_norm/total"] = math.sqrt(sum(v[1] for v in by_kind.values()))
    if hist is not None:
        out["watch/grad_hist"] = [float(x) for x in hist.tolist()]
    return out
