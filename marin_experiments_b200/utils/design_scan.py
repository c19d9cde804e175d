"""Design-space scan for the next MoE run on a B200 box (the role of megagpt-speedrun/design_scan.py
and megagpt-speedrun/decision_table.py, re-derived for B200 memory and throughput).

For a grid of geometries (hidden size D, experts E, experts per token K, expert-width multiple) it
derives the rest of the model with the AdamH heuristic (``optim.heuristic``) and reports, for a fixed
wall-clock budget on one box:

* total and active parameters (``utils.perf_model.param_split`` plus the routed share that is active);
* projected tokens/s from the analytical box model (``utils.perf_model.estimate``), optionally
  rescaled to a measured anchor (a measured tokens/s for one geometry calibrates the model's
  efficiency; the same calibration is applied to every row);
* tokens × total and tokens × active parameters over the budget, relative to a baseline row;
* expert feeding: routed tokens per expert over the run (too few starves the experts);
* per-GPU memory: parameters with fp32 master, gradient and two moments plus the bf16 compute copy
  (18 B each, experts sharded over the expert-parallel group) and activations for one microbatch
  (bytes per token measured on this framework), against the B200's usable HBM.

``decision_table`` ranks measured candidates (tokens/s and a fit verdict from real runs) on
tokens × active parameters, subject to fitting and feeding.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

from ..optim.heuristic import MoeAdamHHeuristic
from .perf_model import Hardware, Layout, estimate, param_split

BYTES_PER_PARAM = 18.0  # fp32 master + fp32 grad + 2 fp32 moments + bf16 compute copy
ACT_BYTES_PER_TOKEN = 2.25e6  # measured: ~36 GB of activations per 16,384 tokens (megagpt geometry)
HBM_BYTES = 178e9  # usable per B200 (torch reports 178.35 GiB total capacity)


@dataclass(frozen=True)
class Candidate:
    name: str
    hidden: int
    experts: int
    k: int
    inter_mult: int = 1


@dataclass
class ScanRow:
    cand: Candidate
    cfg: object
    total: float
    active: float
    tokens_per_s: float
    tokens: float
    tok_x_total: float
    tok_x_active: float
    tokens_per_expert: float
    mem_per_gpu: float

    @property
    def fits(self) -> bool:
        return self.mem_per_gpu <= HBM_BYTES


def build(c: Candidate, seq_len: int = 2048, heuristic: MoeAdamHHeuristic | None = None):
    h = heuristic or MoeAdamHHeuristic()
    cfg = h.build_model_config(c.hidden, seq_len=seq_len, num_experts=c.experts, num_experts_per_token=c.k)
    if c.inter_mult != 1:
        cfg = dataclasses.replace(cfg, intermediate_dim=cfg.intermediate_dim * c.inter_mult)
    return cfg


def params(cfg) -> tuple[float, float]:
    """(total, active) parameters: active counts K of the E routed experts per token."""
    experts, other = param_split(cfg)
    active_experts = experts * cfg.num_experts_per_token / max(cfg.num_experts, 1)
    return experts + other, active_experts + other


def memory_per_gpu(cfg, gpus: int, micro_tokens: int) -> float:
    experts, other = param_split(cfg)
    return BYTES_PER_PARAM * (experts / gpus + other) + ACT_BYTES_PER_TOKEN * micro_tokens


def scan(cands: list[Candidate], *, gpus: int = 8, hours: float = 24.0, tokens_per_gpu: int = 65536,
         micro_tokens: int = 32768, hw: Hardware | None = None, anchor: tuple[object, float] | None = None
         ) -> list[ScanRow]:
    """One row per candidate. ``anchor`` = (model config, measured whole-box tokens/s on this box
    size) rescales every projected tokens/s by measured / modelled for that configuration."""
    scale = 1.0
    if anchor is not None:
        acfg, measured = anchor
        modelled = estimate(acfg, Layout(gpus=gpus, ep=gpus, tokens_per_gpu=tokens_per_gpu), hw).tokens_per_s
        scale = measured / modelled
    rows = []
    for c in cands:
        cfg = build(c)
        total, active = params(cfg)
        tps = scale * estimate(cfg, Layout(gpus=gpus, ep=gpus, tokens_per_gpu=tokens_per_gpu), hw).tokens_per_s
        tokens = tps * hours * 3600
        rows.append(ScanRow(c, cfg, total, active, tps, tokens, tokens * total, tokens * active,
                            tokens * c.k / c.experts, memory_per_gpu(cfg, gpus, micro_tokens)))
    return rows


def table(rows: list[ScanRow], baseline: str | None = None, min_tokens_per_expert: float = 0.0) -> str:
    base = next((r for r in rows if r.cand.name == baseline), rows[0])
    out = ["| name | D | E | K | I | L | total B | active B | tok/s | tokens B | tok×total | tok×active | "
           "tok/expert B | GB/GPU | notes |",
           "|---|---|---|---|---|---|---|---|---|---|---|---|---|---|---|"]
    for r in sorted(rows, key=lambda x: -x.tok_x_total):
        notes = []
        if not r.fits:
            notes.append("does not fit")
        if r.tokens_per_expert < min_tokens_per_expert:
            notes.append("experts starved")
        c = r.cfg
        out.append(f"| {r.cand.name} | {c.hidden_dim} | {c.num_experts} | {c.num_experts_per_token} | "
                   f"{c.intermediate_dim} | {c.num_layers} | {r.total / 1e9:.2f} | {r.active / 1e9:.2f} | "
                   f"{r.tokens_per_s / 1e3:,.0f}K | {r.tokens / 1e9:.1f} | {r.tok_x_total / base.tok_x_total:.2f}x | "
                   f"{r.tok_x_active / base.tok_x_active:.2f}x | {r.tokens_per_expert / 1e9:.3f} | "
                   f"{r.mem_per_gpu / 1e9:.0f} | {', '.join(notes)} |")
    return "\n".join(out)


@dataclass(frozen=True)
class Measured:
    """A real run: whole-box tokens/s (None if it did not run) and whether it fit at full batch."""
    cand: Candidate
    tokens_per_s: float | None
    fit: bool


def decision_table(measured: list[Measured], *, hours: float = 24.0, cooldown_hours: float = 0.0,
                   min_tokens_per_expert: float = 0.0) -> list[tuple[str, float, float, str]]:
    """Rank measured candidates on tokens × active parameters over the pre-training part of the budget
    (``hours - cooldown_hours``). Returns (name, tokens × active, tokens per expert, verdict), best
    first; candidates that did not fit, did not run or starve their experts come last, marked."""
    secs = (hours - cooldown_hours) * 3600
    ranked = []
    for m in measured:
        cfg = build(m.cand)
        _, active = params(cfg)
        if not m.fit or m.tokens_per_s is None:
            ranked.append((m.cand.name, 0.0, 0.0, "does not fit"))
            continue
        tokens = m.tokens_per_s * secs
        tpe = tokens * m.cand.k / m.cand.experts
        verdict = "ok" if tpe >= min_tokens_per_expert else "experts starved"
        ranked.append((m.cand.name, tokens * active, tpe, verdict))
    return sorted(ranked, key=lambda r: (r[3] != "ok", -r[1]))


DEFAULT_CANDIDATES = [
    Candidate("E64/K4", 1536, 64, 4),
    Candidate("E64/K8", 1536, 64, 8),
    Candidate("E128/K8", 1536, 128, 8),
    Candidate("E256/K8", 1536, 256, 8),
    Candidate("E128/K16", 1536, 128, 16),
    Candidate("E64/I x2", 1536, 64, 8, 2),
    Candidate("D2048/E64", 2048, 64, 8),
    Candidate("D2048/E128", 2048, 128, 8),
    Candidate("D2560/E64", 2560, 64, 8),
]


def main():
    from ..parallel.pipeline_entry import megagpt_model

    # calibrated on the measured 8-GPU EP=8 training step of the megagpt geometry (tokens/s)
    rows = scan(DEFAULT_CANDIDATES, anchor=(megagpt_model(), 662_754.0))
    print(table(rows, baseline=DEFAULT_CANDIDATES[0].name))


if __name__ == "__main__":
    main()
