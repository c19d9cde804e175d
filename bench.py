"""Headline benchmark: MoE training tokens/s on the megagpt-speedrun configuration.

Model (random init, bf16 compute, fp32 masters, AdamH): 24 layers, d_model 1536, 16 heads
(head_dim 96), 64 routed experts top-4 with expert d_ff 768 plus one shared expert of d_ff 3072,
vocab 128256, seq 2048, capacity factor 1.25, GatedNorm / QK-norm / XSA / head gate on.
Data: synthetic uniform-random token ids (seed 2). Weak scaling: 64K tokens (32 sequences) per
GPU per step, i.e. 512K tokens per step on 8 GPUs; experts are sharded over all ranks (EP = N).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and a device synchronise,
timed with CUDA events on the compute stream; the reported time is the max over ranks. The step's
working set (12.8 GB of bf16 weights alone) is far larger than the 126 MB L2, so no flush is
needed between steps. The end-to-end figure repeats K steps through ``Trainer.train_step`` with
every step's tokens copied from pinned host memory and the loss read back to the host.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
                       [--config megagpt|grug_dp|adaptive|pp] [--pp-schedule zb|1f1b|gpipe|async]

``--config grug_dp`` (12 layers, d768, 8 experts top-2, seq 1024, 256 sequences per step in total,
pure data parallel) and ``--config adaptive`` (16 layers, d1024, 32 experts with a per-token top-k in
1..8, seq 2048, 256K tokens per step in total, EP = N) are the smaller configurations; their
global batch is fixed, so they scale strongly. ``--config pp`` runs the same architecture as
pipeline stages x expert parallelism (see ``bench_pp``). The default is the headline configuration
above.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

BASELINE_TOK_S = 192000.0  # reference 8xH100 anchor (tokens/s, whole job)
BASELINE_NOTE = ("reference: 192,000 tokens/s for the whole 8xH100 job (24,000 per GPU) on its own anchor "
                 "config (16 layers, seq 4096, top-8, expert d_ff 512): different hardware and config")
METRIC = "MoE train tokens/sec/box at 1/2/4/8 B200; MFU; exposed all-to-all ms/step"
NOMINAL_BF16 = 2.25e15  # dense bf16 tensor peak of one B200 (context only)
FALLBACK_SUSTAINED_BF16 = 1.4e15  # cuBLAS bf16 under the 1 kW power cap, earlier measurement on this hardware


def measured_bf16_peak() -> tuple[float, str]:
    """Sustained cuBLAS bf16 FLOP/s of one GPU from MEASURED_PEAKS.json beside this file (the
    roofline denominator for a kernel timed inside a long step), or the fallback figure."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops_sustained"]) * 1e12, "of measured sustained cuBLAS bf16"
    except (OSError, KeyError, ValueError, TypeError):
        return FALLBACK_SUSTAINED_BF16, "of fallback sustained cuBLAS bf16 (1.4 PFLOP/s)"


def megagpt_config():
    from marin_experiments_b200.config import GrugModelConfig

    return GrugModelConfig(
        vocab_size=128256, hidden_dim=1536, intermediate_dim=768, shared_expert_intermediate_dim=3072,
        num_experts=64, num_experts_per_token=4, num_layers=24, num_heads=16, num_kv_heads=16, head_dim=96,
        max_seq_len=2048, sliding_window=4096, capacity_factor=1.25, router_z_loss_coef=0.001,
    )


# (model config factory, sequences per GPU given the world size, parallelism, scaling, label, default
# microbatch given the world size); "megagpt" is the headline and the default.
def bench_config(name: str, world: int) -> dict:
    from marin_experiments_b200.config import GrugModelConfig

    if name == "megagpt":
        return {"model": megagpt_config(), "seqs_per_gpu": 32, "parallel": "ep", "scaling": "weak",
                "label": "megagpt-speedrun MoE: 24L d1536 16h(hd96) E64 top4 d_ff768 + shared 3072, vocab 128256",
                "micro_batch": 8 if world == 1 else 16, "baseline": BASELINE_TOK_S}
    if name in ("grug_dp", "adaptive"):
        total = 256 if name == "grug_dp" else 128
        if total % world:
            raise ValueError(f"--config {name} keeps {total} sequences per step in total; {world} GPUs do not divide it")
        if name == "adaptive" and 32 % world:
            raise ValueError(f"--config adaptive shards 32 experts over the GPUs; {world} GPUs do not divide them")
    if name == "grug_dp":  # 256 sequences of 1024 per step in total, experts replicated (pure data parallel)
        cfg = GrugModelConfig(vocab_size=128256, hidden_dim=768, intermediate_dim=2048, shared_expert_intermediate_dim=0,
                              num_experts=8, num_experts_per_token=2, num_layers=12, num_heads=12, num_kv_heads=12,
                              head_dim=64, max_seq_len=1024, sliding_window=1024, capacity_factor=1.25,
                              aux_loss_coef=0.01, initializer_std=0.02)
        return {"model": cfg, "seqs_per_gpu": 256 // world, "parallel": "dp", "scaling": "strong",
                "label": "grug MoE: 12L d768 12h(hd64) E8 top2 d_ff2048, vocab 128256, aux LBL 0.01",
                "micro_batch": 32, "baseline": None}
    if name == "adaptive":  # 256K tokens per step in total, per-token top-k in 1..8 by router-score threshold
        cfg = GrugModelConfig(vocab_size=128256, hidden_dim=1024, intermediate_dim=512, shared_expert_intermediate_dim=1024,
                              num_experts=32, num_experts_per_token=8, adaptive_routing=True, min_experts_per_token=1,
                              num_layers=16, num_heads=8, num_kv_heads=8, head_dim=128, max_seq_len=2048,
                              sliding_window=2048, capacity_factor=1.25)
        return {"model": cfg, "seqs_per_gpu": 128 // world, "parallel": "ep", "scaling": "strong",
                "label": "adaptive-sparsity MoE: 16L d1024 8h(hd128) E32 top-k 1..8 d_ff512 + shared 1024, vocab 128256",
                "micro_batch": 16, "baseline": None}
    raise ValueError(f"unknown --config {name!r}")


def flops_per_token(cfg) -> float:
    """Training FLOPs per token: 6 x active matmul parameters + causal attention (fwd+bwd)."""
    d, hd, h, hkv, s = cfg.hidden_dim, cfg.inferred_head_dim, cfg.num_heads, cfg.num_kv_heads, cfg.max_seq_len
    attn_proj = d * (h + 2 * hkv) * hd + h * hd * d + d * h
    gated = 2 * (2 * d * cfg.gated_norm_rank)
    experts = cfg.num_experts_per_token * 3 * d * cfg.intermediate_dim + d * cfg.num_experts
    shared = 3 * d * cfg.shared_expert_intermediate_dim
    per_layer = attn_proj + gated + experts + shared
    head = cfg.vocab_size * cfg.inferred_embed_dim
    dense = cfg.num_layers * per_layer + head + 2 * (2 * d * cfg.gated_norm_rank)
    attn_core = cfg.num_layers * 2 * s * h * hd  # QK^T and PV, causal half, forward
    return 6.0 * dense + 3.0 * attn_core


class ClockSampler:
    """Samples nvidia-smi SM clocks / throttle reasons in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def bench_pp(args) -> int:
    """``--config pp``: pipeline x expert parallelism on the megagpt architecture (24 layers split
    evenly over the stages), PP = N / 2 stages x EP = 2 (PP = N, EP = 1 below 4 GPUs), 16
    microbatches of 8 x 2048 tokens per pipeline replica, delayed-gradient AdamH with staleness 1,
    stage activations over NCCL p2p (isend / irecv, completing in the background). ``--pp-schedule``:
    zb (ZB-H1 zero bubble, default), 1f1b, gpipe (synchronous steps) or async (1F1B without flush,
    one microbatch per tick; a "step" is 16 ticks). Every rank times the same steps with CUDA events;
    the reported time is the max over ranks."""
    import datetime

    import torch.distributed as tdist

    from marin_experiments_b200.config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.ops._ext import check_kernel_errors, ext
    from marin_experiments_b200.optim.delayed import DelayedGrugMoeAdamHConfig
    from marin_experiments_b200.parallel.pipeline import PipelineTrainer, bubble_fraction, init_topology

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    if not tdist.is_initialized():
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), rank=rank, world_size=world,
                                 init_method="env://" if world > 1 else "tcp://127.0.0.1:29599")
    ep = 2 if world >= 4 else 1
    pp = world // ep
    topo = init_topology(pp, ep)
    cfg = megagpt_config()
    import dataclasses

    if args.layers is not None:
        cfg = dataclasses.replace(cfg, num_layers=args.layers)
    opt = DelayedGrugMoeAdamHConfig(tau=1, corrector="none", learning_rate=0.01, adam_lr=6e-4, warmup=0.0)
    run = GrugRunConfig(model=cfg, optimizer=opt, trainer=GrugTrainerConfig(trainer=TrainerConfig(seed=3, num_train_steps=1000)))
    M, mb, seq = 16, 8, cfg.max_seq_len
    sched = args.pp_schedule
    mode = "async" if sched == "async" else "sync"
    pt = PipelineTrainer(run, topo, device=f"cuda:{local_rank}", microbatches=1 if mode == "async" else M,
                         schedule="1f1b" if mode == "async" else sched, mode=mode)
    g = torch.Generator().manual_seed(3 * 1000003 + topo.e)

    def batch(n):
        return {"tokens": torch.randint(0, cfg.vocab_size, (n, seq), generator=g).pin_memory()}

    def one_step(host: bool):
        """One step; returns the last stage's loss as a device tensor (None on other stages)."""
        if mode == "async":
            losses = pt.run_async([batch(mb) for _ in range(M)] if host else [staged_mb[i] for i in range(M)], M,
                                  as_tensors=True)
            return losses[-1] if losses else None
        out = pt.train_step(batch(M * mb) if host else staged_full)
        return out.get("train/cross_entropy_loss")

    staged_full = {"tokens": batch(M * mb)["tokens"].cuda()}
    staged_mb = [{"tokens": batch(mb)["tokens"].cuda()} for _ in range(M)]
    for _ in range(args.warmup):
        one_step(False)
    torch.cuda.synchronize()
    check_kernel_errors()
    clocks = ClockSampler(local_rank)
    tdist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    n0 = ext().launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        one_step(False)
    e1.record()
    torch.cuda.synchronize()
    launches = ext().launch_count() - n0
    tdist.barrier()
    clk = clocks.stop()
    ms_t = torch.tensor([e0.elapsed_time(e1) / args.steps], device="cuda")
    tdist.all_reduce(ms_t, op=tdist.ReduceOp.MAX)
    ms = float(ms_t.item())
    tokens_step = M * mb * seq * ep
    tok_s = tokens_step / (ms / 1e3)
    # end to end: every step's tokens from pinned host memory, loss read back by the last stage
    e2e = None
    if not args.no_e2e:
        tdist.barrier()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(args.steps):
            loss = one_step(True)
            if loss is not None:
                _ = float(loss.item())  # the last stage reads the step's loss back
        a1.record()
        torch.cuda.synchronize()
        et = torch.tensor([a0.elapsed_time(a1) / args.steps], device="cuda")
        tdist.all_reduce(et, op=tdist.ReduceOp.MAX)
        ems = float(et.item())
        e2e = {"value": tokens_step / (ems / 1e3), "unit": "tokens/s", "ms_per_step": ems,
               "h2d_bytes_per_step": M * mb * seq * 8, "d2h_bytes_per_step": 4 if topo.is_last else 0}
    peak = torch.tensor([torch.cuda.max_memory_allocated() / 1e9], device="cuda")
    tdist.all_reduce(peak, op=tdist.ReduceOp.MAX)
    check_kernel_errors()
    fpt = flops_per_token(cfg)
    flop_peak, peak_label = measured_bf16_peak()
    out = {
        "metric": "pipeline-parallel MoE train tokens/sec/box", "value": tok_s, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "tokens_per_s_per_gpu": tok_s / world, "dtype": "bf16",
        "data": "synthetic (uniform random ids, seed 3; random init)",
        "config": {"model": "megagpt-speedrun MoE split into pipeline stages", "name": "pp", "pp": pp, "ep": ep,
                   "schedule": sched, "microbatches": M, "micro_batch": mb, "seq_len": seq, "layers": cfg.num_layers,
                   "tokens_per_step": tokens_step, "optimizer": "delayed AdamH, staleness 1",
                   "parallelism": f"pp{pp}xep{ep}", "l2": "working set >> L2 (no flush needed)",
                   "bubble_model": bubble_fraction("1f1b" if mode == "async" else sched, pp, M)},
        "mfu": tok_s * fpt / (flop_peak * world), "mfu_denominator": f"{flop_peak / 1e12:.1f} TFLOP/s per GPU, {peak_label}",
        "peak_memory_gb": float(peak.item()), "clocks": clk, "gpu_launches": int(launches), "e2e": e2e,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    tdist.barrier()
    tdist.destroy_process_group()
    return 0


def reference_arm(args):
    """The reference is JAX/XLA (jax + levanter + flash-attn-4 + NCCL cu13); none of it is installed in
    this image and there is no network, so its own code path cannot run here."""
    msg = {"impl": "reference", "unavailable": "reference is a JAX/XLA program (jax, marin-levanter, flash-attn-4); "
                                               "jax is not installed in this offline image and baseline/_ref has no "
                                               "runnable JAX stack"}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(msg), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--config", default="megagpt", choices=["megagpt", "grug_dp", "adaptive", "pp"],
                    help="megagpt (headline, weak scaling with EP = N); grug_dp and adaptive: the smaller "
                         "configurations, fixed global batch; pp: pipeline x expert parallelism")
    ap.add_argument("--pp-schedule", default="zb", choices=["zb", "1f1b", "gpipe", "async"])
    ap.add_argument("--seqs-per-gpu", type=int, default=None)
    ap.add_argument("--micro-batch", type=int, default=None,
                    help="sequences per microbatch (gradient accumulation); default 8 on one GPU, where "
                         "~6B parameters with fp32 master, grads and moments leave room for 8 x 2048 tokens of "
                         "activations, and 16 with expert parallelism, where the experts are sharded")
    ap.add_argument("--zero", action="store_true",
                    help="ZeRO: shard the replicated parameters' optimizer state over the ranks (gradient "
                         "reduce-scatter / parameter all-gather over peer memory; MXK_ZERO_P2P=0 for NCCL)")
    ap.add_argument("--remat", default=None, choices=["none", "recompute_all", "save_moe"],
                    help="activation recompute per block (default: none; the model config's value)")
    ap.add_argument("--layers", type=int, default=None, help="(debug only) override layer count")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-trace", default=None,
                    help="after the timed steps, run one more step under torch.profiler, write its Chrome trace "
                         "here and a device-time breakdown by kernel family to <path>.md (shares only)")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return reference_arm(args)
    if args.config == "pp":
        return bench_pp(args)

    from marin_experiments_b200.config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.data.synthetic import UniformTokenBatches
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.parallel import dist as pdist
    from marin_experiments_b200.train.trainer import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    bc = bench_config(args.config, world)
    if args.micro_batch is None:
        args.micro_batch = bc["micro_batch"]
    if args.seqs_per_gpu is None:
        args.seqs_per_gpu = bc["seqs_per_gpu"]
    args.micro_batch = min(args.micro_batch, args.seqs_per_gpu)
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    ep_size = world if bc["parallel"] == "ep" else 1
    if world > 1 and args.zero:
        from marin_experiments_b200.parallel.fsdp import init_zero

        ctx = init_zero(ep_size=ep_size)
    else:
        ctx = pdist.init(ep_size=ep_size) if world > 1 else None
    cfg = bc["model"]
    import dataclasses

    if args.layers is not None:
        cfg = dataclasses.replace(cfg, num_layers=args.layers)
    if args.remat is not None:
        cfg = dataclasses.replace(cfg, remat_mode=args.remat)
    run = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(learning_rate=0.01, adam_lr=6e-4, warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(seed=0, num_train_steps=1000)))
    trainer = Trainer(run, device=f"cuda:{local_rank}", micro_batch=args.micro_batch, dist=ctx)
    if args.config == "megagpt" and world > 1 and args.micro_batch > 8:
        # Guard for the default: one 2048-token sequence of this model keeps ~4.6 GB of activations and
        # exchange buffers (measured on one GPU: 36 GB per 8 sequences). Fall back to 8-sequence
        # microbatches on every rank if any rank lacks the room (same decision everywhere).
        free, _ = torch.cuda.mem_get_info()
        fits = torch.tensor([1.0 if free > args.micro_batch * 4.6e9 * 1.1 else 0.0], device=trainer.device)
        torch.distributed.all_reduce(fits, op=torch.distributed.ReduceOp.MIN)
        if fits.item() < 0.5:
            args.micro_batch = 8
            trainer.micro_batch = 8
    seqs = args.seqs_per_gpu
    seq = cfg.max_seq_len
    data = UniformTokenBatches(seqs, seq, cfg.vocab_size, seed=2, pin=True, rank=rank)

    def barrier():
        if ctx is not None:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        met = trainer.train_step(next(data))
    torch.cuda.synchronize()
    from marin_experiments_b200.ops._ext import check_kernel_errors, ext

    check_kernel_errors()
    # ------------------------------------------------------------------ device-timed steps
    staged = [{"tokens": next(data)["tokens"].to(trainer.device)} for _ in range(args.steps)]
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    clocks = ClockSampler(int(vis[local_rank]) if local_rank < len(vis) and vis[local_rank].strip().isdigit()
                          else local_rank)  # nvidia-smi index of this rank's GPU
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    n0 = ext().launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile = os.environ.get("MXK_PROFILE_TIMED") == "1"  # bracket the timed steps for ncu --profile-from-start off
    if profile:
        torch.cuda.cudart().cudaProfilerStart()
    e0.record()
    for i in range(args.steps):
        met = trainer.train_step(staged[i])
    e1.record()
    torch.cuda.synchronize()
    if profile:
        torch.cuda.cudart().cudaProfilerStop()
    launches = ext().launch_count() - n0
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_t = torch.tensor([ms], device=trainer.device)
    if ctx is not None:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms = float(ms_t.item())
    loss = float(met["train/loss"].item())
    tokens_step = seqs * seq * world
    tok_s = tokens_step / (ms / 1e3)
    fpt = flops_per_token(cfg)
    flop_peak, peak_label = measured_bf16_peak()
    mfu = tok_s * fpt / (flop_peak * world)
    mfu_nominal = tok_s * fpt / (NOMINAL_BF16 * world)
    # ------------------------------------------------------------------ end to end (public API)
    e2e = None
    clk_e2e = None
    if not args.no_e2e:
        host = [next(data) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        clocks_e2e = ClockSampler(clocks.gpu)
        clocks_e2e.start()
        t0 = time.perf_counter()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for i in range(args.steps):
            m = trainer.train_step(host[i])
            _ = float(m["train/loss"].item())
        a1.record()
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / args.steps
        clk_e2e = clocks_e2e.stop()
        ems = a0.elapsed_time(a1) / args.steps
        et = torch.tensor([ems], device=trainer.device)
        if ctx is not None:
            torch.distributed.all_reduce(et, op=torch.distributed.ReduceOp.MAX)
        ems = float(et.item())
        e2e = {"value": tokens_step / (ems / 1e3), "unit": "tokens/s", "ms_per_step": ems, "wall_ms_per_step": wall * 1e3,
               "h2d_bytes_per_step": int(host[0]["tokens"].numel() * host[0]["tokens"].element_size()),
               "d2h_bytes_per_step": 4, "clocks": clk_e2e,
               "ms_x_median_mhz": ems * clk_e2e["sm_mhz"] if clk_e2e.get("sm_mhz") else None}
    # ------------------------------------------- exposed token exchange (one extra, untimed step)
    # Device time spent in the expert-parallel exchange kernels and their cross-rank waits, summed
    # from CUDA events around each exchange (nothing else runs on the stream meanwhile); max over ranks.
    # The same step also times the training stream's gradient synchronisation (the data-parallel
    # all-reduce or ZeRO reduce-scatter / all-gather that backward did not hide).
    exposed = exposed_dp = 0.0
    if ctx is not None:
        from marin_experiments_b200.parallel.dist import dp_timing
        from marin_experiments_b200.parallel.ep import exchange_timing

        barrier()
        with exchange_timing() as xt, dp_timing() as dt:
            trainer.train_step(staged[0])
        xt_t = torch.tensor([xt.ms(), dt.ms()], device=trainer.device)
        torch.distributed.all_reduce(xt_t, op=torch.distributed.ReduceOp.MAX)
        exposed, exposed_dp = (float(v) for v in xt_t.tolist())
    if args.profile_trace:
        from marin_experiments_b200.utils.analysis import breakdown_table, profile_call

        barrier()
        path = args.profile_trace if world == 1 else f"{args.profile_trace}.rank{rank}"
        b = profile_call(lambda: trainer.train_step(staged[0]), steps=1, trace_path=path)
        if rank == 0:
            with open(f"{args.profile_trace}.md", "w") as f:
                f.write(breakdown_table(b) + "\n")
    peak = torch.tensor([torch.cuda.max_memory_allocated() / 1e9], device=trainer.device)  # allocator high-water
    if ctx is not None:
        torch.distributed.all_reduce(peak, op=torch.distributed.ReduceOp.MAX)
    check_kernel_errors()
    out = {
        "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": bc["scaling"],
        "vs_baseline": tok_s / bc["baseline"] if bc["baseline"] else None,
        "vs_baseline_note": BASELINE_NOTE if bc["baseline"] else None,
        "tokens_per_s_per_gpu": tok_s / world,
        "dtype": "bf16", "data": "synthetic (uniform random ids, seed 2; random init)",
        "config": {"model": bc["label"], "name": args.config,
                   "global_batch": seqs * world, "seq_len": seq, "tokens_per_step": tokens_step,
                   "micro_batch": args.micro_batch, "capacity_factor": cfg.capacity_factor,
                   "parallelism": (f"{bc['parallel']}{world}" + ("+zero" if args.zero else "")) if world > 1 else "single", "l2": "working set >> L2 (no flush needed)",
                   "layers": cfg.num_layers, "remat": cfg.remat_mode, "zero": bool(args.zero and world > 1),
                   "ep_shared_overlap": bool(world > 1 and cfg.num_experts > 0 and ep_size > 1
                                             and os.environ.get("MXK_EP_OVERLAP", "1") == "1"
                                             and os.environ.get("MXK_EP_IMPL", "peer") == "peer")},
        "mfu": mfu, "mfu_denominator": f"{flop_peak / 1e12:.1f} TFLOP/s per GPU, {peak_label}",
        "mfu_nominal": mfu_nominal, "mfu_nominal_denominator": "2250 TFLOP/s per GPU, nominal dense bf16",
        "ms_x_median_mhz": ms * clk["sm_mhz"] if clk.get("sm_mhz") else None,
        "exposed_all_to_all_ms_per_step": exposed, "exposed_dp_sync_ms_per_step": exposed_dp, "peak_memory_gb": float(peak.item()), "flops_per_token": fpt, "loss": loss,
        "clocks": clk, "gpu_launches": int(launches),
        "e2e": e2e,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    if ctx is not None:
        pdist.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
