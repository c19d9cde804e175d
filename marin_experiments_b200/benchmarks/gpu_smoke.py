"""Pipeline-stage smoke on one GPU (grug-moe-pp/gpu_smoke.py:44-124, megagpt-speedrun/train_pp.py
gpu_smoke): build each pipeline stage of a model in turn on the GPU, run one forward + backward of a
microbatch through it, and report the stage's time and peak memory -- a check that every stage of
a PP layout fits and runs before launching the multi-GPU job.

Run: ``python -m marin_experiments_b200.benchmarks.gpu_smoke [--pp 4] [--layers 24] [--mb 8]``.
"""

from __future__ import annotations

import argparse
import json

import torch


def run(pp: int = 4, layers: int = 24, mb: int = 8, seq: int = 2048):
    from marin_experiments_b200.config import GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.ops._ext import check_kernel_errors
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.parallel.pipeline import stage_layers
    from marin_experiments_b200.parallel.pipeline_entry import megagpt_model
    from marin_experiments_b200.train.trainer import Trainer

    cfg = megagpt_model(layers, seq)
    out = []
    tok = torch.randint(0, cfg.vocab_size, (mb, seq), device="cuda")
    for s in range(pp):
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        run_cfg = GrugRunConfig(model=cfg, optimizer=GrugMoeAdamHConfig(warmup=0.0),
                                trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10)))
        tr = Trainer(run_cfg, device="cuda", model_kwargs=dict(layers=stage_layers(layers, pp, s),
                                                               with_embed=s == 0, with_head=s == pp - 1))
        m = tr.model
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        x = m.embed(tok) if s == 0 else torch.randn(mb * seq, cfg.hidden_dim, device="cuda").bfloat16().requires_grad_()
        h, stats = m.body(x, mb, seq)
        if s == pp - 1:
            y = m.head_input(h).float().square().mean()
        else:
            y = h.float().square().mean()
        y.backward()
        e1.record()
        torch.cuda.synchronize()
        check_kernel_errors()
        out.append({"stage": s, "layers": list(stage_layers(layers, pp, s))[::max(1, layers // pp - 1)],
                    "fwd_bwd_ms": e0.elapsed_time(e1), "peak_gib": torch.cuda.max_memory_allocated() / 2 ** 30})
        del tr, m, x, h, y
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--pp", type=int, default=4)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--mb", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    a = ap.parse_args()
    run(a.pp, a.layers, a.mb, a.seq)
