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

``pp_from_profile`` predicts pipeline parallelism from a measured expert-parallel step (the
profile-anchored method of megagpt-speedrun/h100_pp_model.py), and ``cross_node`` compares
synchronous data parallelism with pipeline parallelism across nodes joined by per-GPU network
interfaces (the question of delayed-gradient-pp/pp_throughput_model.py).

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


# ------------------------------------------------------------------ profile-anchored PP prediction
@dataclass(frozen=True)
class StepProfile:
    """A measured expert-parallel training step, split into additive device-time parts (ms):
    ``compute`` (everything that is not the two below), ``ep_exposed`` (device time inside the token
    exchanges, ``bench.py``'s exposed all-to-all), ``optimizer`` (the fused optimizer passes)."""
    step_ms: float
    ep_exposed_ms: float
    optimizer_ms: float
    tokens_per_gpu: int = 65536

    @property
    def compute_ms(self) -> float:
        return self.step_ms - self.ep_exposed_ms - self.optimizer_ms


@dataclass(frozen=True)
class PPKnobs:
    """The uncertain parts of a pipeline-parallel prediction. ``eta_sync``: GEMM efficiency of the
    smaller per-microbatch GEMMs of a synchronous schedule (1 = as efficient as the measured step);
    ``eta_async``: the same for the no-flush asynchronous schedule, whose stages run whole batches;
    ``recompute``: compute multiplier for activation recompute; ``token_tax``: extra tokens the
    asynchronous schedule's staleness costs to reach the same loss (a fraction)."""
    eta_sync: float = 0.9
    eta_async: float = 1.0
    recompute: float = 1.0
    token_tax: float = 0.0


def pp_from_profile(cfg, prof: StepProfile, *, stages: int, microbatches: int, schedule: str = "1f1b",
                    knobs: PPKnobs = PPKnobs(), hw: Hardware | None = None) -> dict:
    """Per-GPU step time of pipeline parallelism on the same GPUs, from a measured EP step.

    PP keeps each layer's experts on its stage's GPU, so the token exchange disappears; what is
    added: the stage-boundary activation sends over NVLink (forward activation and backward gradient
    per microbatch, ``tokens * D * 2`` bytes each way per boundary, overlapped except for the
    pipeline fill), the schedule's bubble (``parallel.schedules`` simulator) for the synchronous
    schedules, and the knobs. The optimizer part is kept (same parameters per GPU in total).
    Returns step times (ms), tokens/s of the job and the speed-up over the measured step, for the
    synchronous schedule and the asynchronous one (effective tokens/s after the token tax)."""
    from ..parallel.schedules import SCHEDULES, simulate

    hw = hw or Hardware.measured()
    act = prof.tokens_per_gpu * cfg.hidden_dim * 2  # one direction, per step, per boundary
    p2p_ms = 2 * act / hw.nvlink_bytes_s * 1e3 / microbatches  # the fill / drain part that stays exposed
    sched = SCHEDULES[schedule](stages, microbatches)
    sim = simulate(sched, 1.0, 1.0, 1.0) if schedule == "zb" else simulate(sched, 1.0, 2.0)
    bubble = sim["bubble"]
    sync_busy = prof.compute_ms / knobs.eta_sync * knobs.recompute
    sync_ms = sync_busy / (1 - bubble) + p2p_ms + prof.optimizer_ms
    async_ms = prof.compute_ms / knobs.eta_async + p2p_ms + prof.optimizer_ms
    n_tok = prof.tokens_per_gpu
    return {
        "ep_ms": prof.step_ms, "sync_ms": sync_ms, "async_ms": async_ms, "bubble": bubble, "p2p_ms": p2p_ms,
        "ep_tok_s_per_gpu": n_tok / prof.step_ms * 1e3,
        "sync_tok_s_per_gpu": n_tok / sync_ms * 1e3,
        "async_tok_s_per_gpu": n_tok / async_ms * 1e3 / (1 + knobs.token_tax),
        "sync_speedup": prof.step_ms / sync_ms,
        "async_speedup": prof.step_ms / async_ms / (1 + knobs.token_tax),
    }


# ------------------------------------------------------------------ across nodes
@dataclass(frozen=True)
class Cluster:
    """Nodes of ``gpus_per_node`` NVSwitch-connected GPUs joined by a per-GPU network interface of
    ``net_bytes_s`` each way (400 Gb/s per GPU: 50 GB/s); ``net_overlap`` of the cross-node gradient
    all-reduce hides under the backward pass."""
    nodes: int = 2
    gpus_per_node: int = 8
    net_bytes_s: float = 50e9
    net_overlap: float = 0.5


def cross_node(cfg, cl: Cluster, *, tokens_per_gpu: int = 65536, microbatches: int = 8, schedule: str = "1f1b",
               hw: Hardware | None = None) -> dict:
    """Synchronous data parallelism across nodes (expert parallelism inside each node) vs pipeline
    parallelism across nodes (one stage per node, expert parallelism inside it).

    DP: every step all-reduces the fp32 gradients across nodes: each GPU carries its expert shard and
    1/gpus_per_node of the replicated parameters (reduced inside the node first), ``2 (n-1)/n`` of
    that through its own interface, all GPUs of a node in parallel. PP: only the stage-boundary activations (forward) and their
    gradients (backward) cross the network, ``tokens * D * 2`` bytes each way per GPU, overlapped
    except for the fill, plus the schedule's bubble. The in-node part of both is ``estimate`` for one
    node. Returns step times (s), tokens/s of the cluster, and the ratio of the cross-node
    communication to the compute (above 1 the network is the bound: the regime where PP pays)."""
    from ..parallel.schedules import SCHEDULES, simulate

    hw = hw or Hardware.measured()
    node = estimate(cfg, Layout(gpus=cl.gpus_per_node, ep=cl.gpus_per_node, tokens_per_gpu=tokens_per_gpu), hw)
    n = cl.nodes
    experts, other = param_split(cfg)
    # per GPU across the network: its own expert shard, and 1/gpus_per_node of the replicated
    # parameters (reduced inside the node over NVLink first); each GPU's interface carries its share
    shard = (experts + other) * 4 / cl.gpus_per_node
    dp_net = 2 * (n - 1) / n * shard / cl.net_bytes_s if n > 1 else 0.0
    dp_step = node.step_s + (1 - cl.net_overlap) * dp_net
    act = tokens_per_gpu * cfg.hidden_dim * 2
    pp_net = 2 * act / cl.net_bytes_s
    bubble = 0.0
    if n > 1:
        sched = SCHEDULES[schedule](n, microbatches)
        sim = simulate(sched, 1.0, 1.0, 1.0) if schedule == "zb" else simulate(sched, 1.0, 2.0)
        bubble = sim["bubble"]
    # a stage holds 1/n of the layers: its per-step compute is the node's for 1/n of the model on n x
    # the tokens per GPU, i.e. the same busy time; the network part overlaps except the fill
    pp_step = node.step_s / (1 - bubble) + pp_net / microbatches
    total = cl.nodes * cl.gpus_per_node * tokens_per_gpu
    return {"dp_step_s": dp_step, "pp_step_s": pp_step, "dp_tok_s": total / dp_step, "pp_tok_s": total / pp_step,
            "dp_net_s": dp_net, "pp_net_s": pp_net, "bubble": bubble,
            "dp_comm_compute_ratio": dp_net / node.parts["compute_s"],
            "pp_comm_compute_ratio": pp_net / node.parts["compute_s"]}


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
    # the measured 4-GPU EP step (731.9 ms, 131.6 ms exposed exchange, ~43 ms optimizer)
    prof = StepProfile(step_ms=731.9, ep_exposed_ms=131.6, optimizer_ms=43.0)
    for sched in ("1f1b", "zb"):
        r = pp_from_profile(cfg, prof, stages=4, microbatches=16, schedule=sched)
        print(f"PP4 {sched}: sync {r['sync_ms']:.0f} ms ({r['sync_speedup']:.2f}x), "
              f"async {r['async_ms']:.0f} ms ({r['async_speedup']:.2f}x), bubble {r['bubble']:.3f}")
    for nodes in (2, 4, 8):
        r = cross_node(cfg, Cluster(nodes=nodes))
        print(f"{nodes} nodes: DP {r['dp_tok_s']:,.0f} tok/s, PP {r['pp_tok_s']:,.0f} tok/s, "
              f"network/compute DP {r['dp_comm_compute_ratio']:.2f} PP {r['pp_comm_compute_ratio']:.3f}")


if __name__ == "__main__":
    main()
