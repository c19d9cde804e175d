"""Pipeline-parallel entry points (megagpt-speedrun/train_pp.py:166-553): ``run_pp_sync`` and
``run_pp_async``, launched one process per GPU (``torchrun --nproc-per-node N``).

Environment: ``SP_PP`` (stages, default world size / ``SP_PP_EP``), ``SP_PP_EP`` (expert-parallel ranks
per stage, default 1), ``SP_PP_SCHEDULE`` (``gpipe`` | ``1f1b`` | ``zb``, sync only), ``SP_MICRO``
(microbatches per step, default 16), ``SP_MB`` (sequences per microbatch, default 8), ``SP_SEQ``,
``SP_STEPS``, ``SP_WARMUP_STEPS``, ``SP_LAYERS`` (default 24), ``SP_HIDDEN`` (heads follow at head dim
96), ``SP_EXPERTS``, ``SP_TOPK``, ``SP_VOCAB`` over the megagpt config (d_model 1536, 16 heads, 64
experts top-4 of width 768 + shared 3072; the ``MOE_PP_*`` names of the pipeline benchmark are
accepted as aliases: STAGE, EP, NMICRO, MICROBATCH, SEQ, LAYERS, HIDDEN, EXPERTS, EPT, VOCAB),
``SP_DELAY_TAU`` (sync:
0; async: the delayed-gradient optimizer with per-stage staleness). Each measured step prints
``[PP_THRUPUT] step=N dt=...s tok_s=... bubble_model=...`` on the last stage.
"""

from __future__ import annotations

import dataclasses
import datetime
import os
import time

import torch
import torch.distributed as tdist

from ..config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
from .pipeline import PipelineTrainer, async_stage_delay, bubble_fraction, init_topology


# The pipeline benchmark's names (grug-moe-pp/benchmark.py:369-389) are accepted as aliases.
_ALIASES = {"SP_PP": "MOE_PP_STAGE", "SP_PP_EP": "MOE_PP_EP", "SP_MICRO": "MOE_PP_NMICRO", "SP_MB": "MOE_PP_MICROBATCH",
            "SP_SEQ": "MOE_PP_SEQ", "SP_LAYERS": "MOE_PP_LAYERS", "SP_HIDDEN": "MOE_PP_HIDDEN",
            "SP_EXPERTS": "MOE_PP_EXPERTS", "SP_TOPK": "MOE_PP_EPT", "SP_VOCAB": "MOE_PP_VOCAB"}


def _env(k, d):
    v = os.environ.get(k, "") or os.environ.get(_ALIASES.get(k, ""), "")
    return v if v else d


def megagpt_model(layers: int = 24, seq: int = 2048) -> GrugModelConfig:
    return GrugModelConfig(vocab_size=128256, hidden_dim=1536, intermediate_dim=768,
                           shared_expert_intermediate_dim=3072, num_experts=64, num_experts_per_token=4,
                           num_layers=layers, num_heads=16, num_kv_heads=16, head_dim=96, max_seq_len=seq,
                           sliding_window=seq, capacity_factor=1.25)


def _setup():
    if not tdist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        tdist.init_process_group(backend, timeout=datetime.timedelta(seconds=float(_env("SP_PG_TIMEOUT", "300"))))
    if torch.cuda.is_available():
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _config(delayed: bool, pp: int, stage: int):
    from ..optim import GrugMoeAdamHConfig
    from ..optim.delayed import DelayedGrugMoeAdamHConfig

    model = megagpt_model(int(_env("SP_LAYERS", "24")), int(_env("SP_SEQ", "2048")))
    hidden = int(_env("SP_HIDDEN", str(model.hidden_dim)))
    if hidden != model.hidden_dim:  # keep the head dim (96): heads follow the width
        model = dataclasses.replace(model, hidden_dim=hidden, num_heads=max(1, hidden // 96),
                                    num_kv_heads=max(1, hidden // 96))
    model = dataclasses.replace(model, num_experts=int(_env("SP_EXPERTS", str(model.num_experts))),
                                num_experts_per_token=int(_env("SP_TOPK", str(model.num_experts_per_token))),
                                vocab_size=int(_env("SP_VOCAB", str(model.vocab_size))))
    if delayed:
        opt = DelayedGrugMoeAdamHConfig(tau=int(_env("SP_DELAY_TAU", str(async_stage_delay(pp, stage)))),
                                        corrector=_env("SP_DELAY_CORRECTOR", "none"), warmup=0.0)
    else:
        opt = GrugMoeAdamHConfig(warmup=0.0)
    return GrugRunConfig(model=model, optimizer=opt,
                         trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=1000, seed=3)))


def _batches(n, mb, seq, vocab, seed, device_rank):
    g = torch.Generator().manual_seed(seed * 1000003 + device_rank)
    for _ in range(n):
        t = torch.randint(0, vocab, (mb, seq), generator=g)
        yield {"tokens": t.pin_memory() if torch.cuda.is_available() else t}


def run_pp_sync() -> dict | None:
    dev = _setup()
    world = tdist.get_world_size()
    ep = int(_env("SP_PP_EP", "1"))
    pp = int(_env("SP_PP", str(world // ep)))
    topo = init_topology(pp, ep)
    M, mb = int(_env("SP_MICRO", "16")), int(_env("SP_MB", "8"))
    sched = _env("SP_PP_SCHEDULE", "1f1b")
    cfg = _config(False, pp, topo.stage)
    pt = PipelineTrainer(cfg, topo, device=dev, microbatches=M, schedule=sched, mode="sync",
                         zero=_env("SP_PP_ZERO", "0") == "1")
    steps, warm = int(_env("SP_STEPS", "4")), int(_env("SP_WARMUP_STEPS", "2"))
    seq = cfg.model.max_seq_len
    data = list(_batches(steps + warm, M * mb, seq, cfg.model.vocab_size, 3, topo.e))
    res = None
    for i, b in enumerate(data):
        if i == warm:
            tdist.barrier()
            if dev.type == "cuda":
                torch.cuda.synchronize()
            t0 = time.perf_counter()
        out = pt.train_step(b)
    tdist.barrier()
    if dev.type == "cuda":
        torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / steps
    tokens = M * mb * seq * ep  # one pipeline replica per expert-parallel index
    if topo.is_last and topo.e == 0:
        res = {"tok_s": tokens / dt, "step_s": dt, "schedule": sched, "pp": pp, "ep": ep,
               "bubble_model": bubble_fraction(sched, pp, M), "loss": float(out["train/cross_entropy_loss"])}
        print(f"[PP_THRUPUT] steps={steps} dt={dt:.3f}s tok_s={res['tok_s']:.0f} schedule={sched} pp={pp} ep={ep} "
              f"bubble_model={res['bubble_model']:.3f} loss={res['loss']:.4f}", flush=True)
    tdist.barrier()
    tdist.destroy_process_group()
    return res


def run_pp_async() -> dict | None:
    dev = _setup()
    world = tdist.get_world_size()
    ep = int(_env("SP_PP_EP", "1"))
    pp = int(_env("SP_PP", str(world // ep)))
    topo = init_topology(pp, ep)
    mb = int(_env("SP_MB", "8"))
    cfg = _config(True, pp, topo.stage)
    pt = PipelineTrainer(cfg, topo, device=dev, microbatches=1, mode="async", zero=_env("SP_PP_ZERO", "0") == "1")
    warm_ticks, ticks = int(_env("SP_WARMUP_TICKS", str(2 * pp))), int(_env("SP_TICKS", "16"))
    seq = cfg.model.max_seq_len
    pt.run_async(_batches(warm_ticks, mb, seq, cfg.model.vocab_size, 3, topo.e), warm_ticks)
    tdist.barrier()
    if dev.type == "cuda":
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    losses = pt.run_async(_batches(ticks, mb, seq, cfg.model.vocab_size, 4, topo.e), ticks)
    tdist.barrier()
    if dev.type == "cuda":
        torch.cuda.synchronize()
    el = time.perf_counter() - t0
    res = None
    if topo.is_last and topo.e == 0:
        res = {"tok_s": ticks * mb * seq * ep / el, "elapsed_s": el, "ticks": ticks, "loss": losses[-1]}
        print(f"[PP_THRUPUT] ticks={ticks} elapsed={el:.2f}s tok_s={res['tok_s']:.0f} pp={pp} ep={ep} "
              f"loss={losses[-1]:.4f}", flush=True)
    tdist.barrier()
    tdist.destroy_process_group()
    return res


if __name__ == "__main__":
    (run_pp_async if _env("SP_PP_MODE", "sync") == "async" else run_pp_sync)()
