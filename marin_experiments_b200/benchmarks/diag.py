"""Diagnostic side entries of the launcher (``SP_DIAG=ragged|ring|fit|attn``).

The reference's launcher has the same four side entries (megagpt-speedrun/_diag_ragged.py:26-317,
reached through ``SP_DIAG`` in megagpt-speedrun/launch.py), written to isolate an XLA fallback in
its grouped matmul and to test whether a configuration fits. Here they answer the same questions
about this framework's own kernels, each printing one JSON line per measurement:

* ``ragged``: the grouped expert GEMMs (forward with the SwiGLU epilogue, input gradients, fp32
  weight gradients) at the expert shapes, against ``torch.bmm``, with the peak device memory;
* ``ring``: one expert-parallel MoE layer (token exchange inside the kernels + grouped GEMMs)
  forward and backward on the ranks of ``torchrun``, device time per iteration (max over ranks)
  and peak memory;
* ``fit``: one training step of the megagpt model at a microbatch (``SP_DIAG_MB``, default 8 sequences),
  the peak device memory and the allocator report of ``utils.memory``;
* ``attn``: the attention forward / backward benchmark.
"""

from __future__ import annotations

import json
import os
import sys

import torch


def ragged() -> list[dict]:
    from . import gemm_bench

    shapes = [s for s in gemm_bench.SHAPES if s[4] in ("gfwd", "gdx", "gdw")]
    torch.cuda.reset_peak_memory_stats()
    rows = gemm_bench.run(shapes)
    peak = torch.cuda.max_memory_allocated() / 1e9
    print(json.dumps({"diag": "ragged", "peak_memory_gb": peak}), flush=True)
    return rows


def ring(t: int = 32768, iters: int = 5) -> dict:
    import datetime

    import torch.distributed as dist

    from ..config import GrugModelConfig
    from ..ops import api
    from ..parallel import ep
    from ..parallel.pipeline_entry import megagpt_model

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        cfg: GrugModelConfig = megagpt_model()
        dev = torch.device("cuda", torch.cuda.current_device())
        e, k, d, inter = cfg.num_experts, cfg.num_experts_per_token, cfg.hidden_dim, cfg.intermediate_dim
        e_loc = e // world
        g = torch.Generator(device="cuda").manual_seed(rank)
        x = (torch.randn(t, d, device=dev, generator=g) * 0.5).bfloat16().requires_grad_(True)
        wr = (torch.randn(e, d, device=dev, generator=g) / 16).bfloat16()
        wgu = (torch.randn(e_loc, 2 * inter, d, device=dev, generator=g) / 32).bfloat16()
        wdn = (torch.randn(e_loc, d, inter, device=dev, generator=g) / 32).bfloat16()
        for w in (wgu, wdn):
            w.main_grad = torch.zeros(w.shape, dtype=torch.float32, device=dev)
        wr.main_grad = torch.zeros(wr.shape, dtype=torch.float32, device=dev)
        gy = torch.randn(t, d, device=dev, generator=g).bfloat16()
        cap = api.capacity_for(t, k, e, cfg.capacity_factor)

        def step():
            r = api.route(x, wr, torch.zeros(e, device=dev), k, qb_count=max(1, t * k // e))
            y = ep.moe_experts_ep(x, r, wgu, wdn, cap, dist.group.WORLD, residual=x)
            y.backward(gy)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            step()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / iters, torch.cuda.max_memory_allocated() / 1e9], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        out = {"diag": "ring", "ep": world, "tokens_per_rank": t, "ms_per_layer_fwd_bwd": float(ms[0]),
               "peak_memory_gb": float(ms[1]), "impl": ep.ep_impl()}
        if rank == 0:
            print(json.dumps(out), flush=True)
        return out
    finally:
        dist.destroy_process_group()


def fit(micro_batch: int | None = None, seqs: int = 32) -> dict:
    from ..config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from ..data.synthetic import UniformTokenBatches
    from ..optim import GrugMoeAdamHConfig
    from ..parallel.pipeline_entry import megagpt_model
    from ..train.trainer import Trainer
    from ..utils.memory import memory_report

    mb = micro_batch or int(os.environ.get("SP_DIAG_MB", "8"))
    cfg = megagpt_model()
    run = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(learning_rate=0.01, adam_lr=6e-4, warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(seed=0, num_train_steps=10)))
    tr = Trainer(run, device="cuda", micro_batch=mb)
    data = UniformTokenBatches(seqs, cfg.max_seq_len, cfg.vocab_size, seed=0, pin=True)
    torch.cuda.reset_peak_memory_stats()
    out = {"diag": "fit", "micro_batch": mb, "fits": True}
    try:
        tr.train_step(next(data))
        torch.cuda.synchronize()
    except torch.OutOfMemoryError as exc:
        out.update(fits=False, error=str(exc).splitlines()[0])
    out["peak_memory_gb"] = torch.cuda.max_memory_allocated() / 1e9
    out["total_memory_gb"] = torch.cuda.get_device_properties(0).total_memory / 1e9
    print(json.dumps(out), flush=True)
    print(memory_report(n=8), flush=True)
    return out


def attn() -> None:
    from . import attn_bench

    attn_bench.run()


MODES = {"ragged": ragged, "ring": ring, "fit": fit, "attn": attn}


def main(mode: str | None = None) -> None:
    mode = mode or os.environ.get("SP_DIAG", "")
    if mode not in MODES:
        raise SystemExit(f"SP_DIAG must be one of {sorted(MODES)}, got {mode!r}")
    MODES[mode]()


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
