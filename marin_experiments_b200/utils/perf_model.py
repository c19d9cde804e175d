"""Analytical throughput model of MoE training on a B200 box (the role of
megagpt-speedrun/h100_pp_model.py:23-119 and delayed-gradient-pp/pp_throughput_model.py:41-222,
re-derived for one NVSwitch node).

Per optimizer step and per GPU it estimates:

* compute: training FLOPs (``utils.flops.training_flops_per_token``) at the measured sustained bf16
  GEMM rate times a realised efficiency;
* expert-parallel exchange: 4 row exchanges per MoE layer per microbatch (dispatch and combine,
  forward and backward), ``tokens * K * D * 2`` bytes each, the ``(W-1)/W`` remote share at the
  measured NVLink peer bandwidth, partly hidden (``ep_overlap``);
* data-parallel gradient all-reduce of the replicated parameters (ring, ``2 (n-1)/n`` of the fp32
  bytes at the measured all-reduce bus bandwidth), partly hidden;
* pipeline bubble from the schedule simulator (``parallel.schedules``);
* the optimizer pass: ~48 bytes of HBM traffic per fp32 parameter held by the GPU.

Peaks come from ``MEASURED_PEAKS.json`` at the repository root when present (written by the
benchmark driver of the machine), else from the constants below.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field, replace

from .flops import training_flops_per_token

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


@dataclass(frozen=True)
class Hardware:
    bf16_flops: float = 1.35e15  # sustained dense bf16 GEMM rate under the power cap
    hbm_bytes_s: float = 6.5e12
    nvlink_bytes_s: float = 770e9  # peer copy, per direction per GPU
    allreduce_bus_bytes_s: float = 725e9  # 8-rank NCCL all-reduce bus bandwidth at 1 GiB
    gemm_efficiency: float = 0.55  # realised fraction of the GEMM rate over a whole step
    gpus_per_node: int = 8

    @staticmethod
    def measured(path: str | None = None) -> "Hardware":
        path = path or os.path.join(_ROOT, "MEASURED_PEAKS.json")
        hw = Hardware()
        try:
            with open(path) as f:
                m = json.load(f)
        except (OSError, ValueError):
            return hw
        if m.get("bf16_tflops_sustained"):
            hw = replace(hw, bf16_flops=float(m["bf16_tflops_sustained"]) * 1e12)
        if m.get("hbm_gbs"):
            hw = replace(hw, hbm_bytes_s=float(m["hbm_gbs"]) * 1e9)
        return hw


@dataclass(frozen=True)
class Layout:
    gpus: int = 8
    ep: int = 8
    pp: int = 1
    tp: int = 1
    tokens_per_gpu: int = 65536  # per optimizer step
    microbatches: int = 4
    schedule: str = "1f1b"
    ep_overlap: float = 0.0  # fraction of the EP exchange hidden under compute
    dp_overlap: float = 0.5


@dataclass
class Estimate:
    step_s: float
    tokens_per_s: float
    mfu: float
    parts: dict = field(default_factory=dict)

    @property
    def exposed_comm_fraction(self) -> float:
        comm = self.parts.get("ep_exposed_s", 0.0) + self.parts.get("dp_exposed_s", 0.0)
        return comm / self.step_s if self.step_s else 0.0


def param_split(cfg) -> tuple[float, float]:
    """(routed expert parameters, everything else)."""
    mats = 3 if cfg.glu else 2
    experts = cfg.num_layers * cfg.num_experts * mats * cfg.hidden_dim * cfg.intermediate_dim if cfg.is_moe else 0
    d, hd = cfg.hidden_dim, cfg.inferred_head_dim
    attn = cfg.num_layers * (d * hd * (2 * cfg.num_heads + 2 * cfg.num_kv_heads) + cfg.num_heads * d)
    shared = cfg.num_layers * mats * d * (cfg.shared_expert_intermediate_dim if cfg.is_moe else cfg.intermediate_dim)
    router = cfg.num_layers * d * cfg.num_experts if cfg.is_moe else 0
    emb = cfg.vocab_size * cfg.inferred_embed_dim * (1 if cfg.tie_embeddings else 2)
    return float(experts), float(attn + shared + router + emb)


def estimate(cfg, layout: Layout, hw: Hardware | None = None) -> Estimate:
    from ..parallel.schedules import SCHEDULES, simulate

    hw = hw or Hardware.measured()
    n = layout.gpus
    toks = layout.tokens_per_gpu
    fpt = training_flops_per_token(cfg)
    # tokens_per_gpu = step tokens / gpus: per-GPU work is the same under DP, EP, PP and TP
    compute = fpt * toks / (hw.bf16_flops * hw.gemm_efficiency)
    parts = {"compute_s": compute}
    ep_s = 0.0
    if cfg.is_moe and layout.ep > 1:
        layers = cfg.num_layers / layout.pp
        bytes_ = 4 * layers * toks * cfg.num_experts_per_token * cfg.hidden_dim * 2 * (layout.ep - 1) / layout.ep
        ep_s = bytes_ / hw.nvlink_bytes_s
    parts["ep_exchange_s"] = ep_s
    parts["ep_exposed_s"] = ep_s * (1 - layout.ep_overlap)
    experts, other = param_split(cfg)
    dp = n // (layout.ep * layout.pp * layout.tp) if cfg.is_moe else n // (layout.pp * layout.tp)
    replicas_of_other = n // (layout.pp * layout.tp)
    dp_s = 0.0
    if replicas_of_other > 1:
        vol = other / (layout.pp * layout.tp) * 4
        dp_s += 2 * (replicas_of_other - 1) / replicas_of_other * vol / hw.allreduce_bus_bytes_s
    if cfg.is_moe and dp > 1:
        vol = experts / (layout.ep * layout.pp) * 4
        dp_s += 2 * (dp - 1) / dp * vol / hw.allreduce_bus_bytes_s
    parts["dp_allreduce_s"] = dp_s
    parts["dp_exposed_s"] = dp_s * (1 - layout.dp_overlap)
    held = (experts / (layout.ep * layout.pp) if cfg.is_moe else 0) + other / (layout.pp * layout.tp)
    parts["optimizer_s"] = held * 48 / hw.hbm_bytes_s
    bubble = 0.0
    if layout.pp > 1:
        sched = SCHEDULES[layout.schedule](layout.pp, layout.microbatches)
        sim = simulate(sched, 1.0, 1.0, 1.0) if layout.schedule == "zb" else simulate(sched, 1.0, 2.0)
        bubble = sim["bubble"]
    parts["pp_bubble_fraction"] = bubble
    busy = compute + parts["ep_exposed_s"]
    step = busy / (1 - bubble) + parts["dp_exposed_s"] + parts["optimizer_s"]
    tok_s = toks * n / step
    mfu = tok_s * fpt / (n * 2.25e15)
    return Estimate(step, tok_s, mfu, parts)


def table(cfg, layouts: list[Layout], hw: Hardware | None = None) -> str:
    rows = ["| gpus | ep | pp | tp | sched | step ms | tok/s | MFU | exposed comm |", "|---|---|---|---|---|---|---|---|---|"]
    for lay in layouts:
        e = estimate(cfg, lay, hw)
        rows.append(f"| {lay.gpus} | {lay.ep} | {lay.pp} | {lay.tp} | {lay.schedule} | {e.step_s * 1e3:.1f} | "
                    f"{e.tokens_per_s:,.0f} | {e.mfu:.3f} | {e.exposed_comm_fraction:.3f} |")
    return "\n".join(rows)


def main():
    from ..parallel.pipeline_entry import megagpt_model

    cfg = megagpt_model()
    lays = [Layout(gpus=g, ep=g) for g in (1, 2, 4, 8)]
    lays += [Layout(gpus=8, ep=2, pp=4, microbatches=16, schedule=s) for s in ("gpipe", "1f1b", "zb")]
    print(table(cfg, lays))


if __name__ == "__main__":
    main()
