"""Neighbour-exchange bandwidth probe (grug-moe-pp/ppermute_probe.py): every rank sends a buffer to
rank + 1 and receives one from rank - 1 (the pipeline-stage transfer pattern), at a ladder of sizes,
over the process group's backend (NCCL over NVLink on GPUs, gloo on the CPU). Each size reports the
time per exchange (max over ranks; CUDA events on GPUs, wall clock on the CPU) and the bandwidth per
direction, which for NVLink peers sits against the measured 770 GB/s peer copy.

Run: ``python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m
marin_experiments_b200.benchmarks.p2p_probe [--sizes-mb 1,16,256] [--iters 10]`` (rank 0 prints one
JSON line per size).
"""

from __future__ import annotations

import argparse
import datetime
import json
import time

import torch
import torch.distributed as dist


def exchange(buf: torch.Tensor, out: torch.Tensor) -> None:
    r, w = dist.get_rank(), dist.get_world_size()
    ops = [dist.P2POp(dist.isend, buf, (r + 1) % w), dist.P2POp(dist.irecv, out, (r - 1) % w)]
    for req in dist.batch_isend_irecv(ops):
        req.wait()


def probe(sizes_mb=(1, 16, 256), iters: int = 10, warmup: int = 2) -> list[dict]:
    dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    rows = []
    for mb in sizes_mb:
        n = int(mb * (1 << 20)) // 4
        buf = torch.full((n,), float(dist.get_rank()), device=dev)
        out = torch.empty_like(buf)
        for _ in range(warmup):
            exchange(buf, out)
        if float(out[0]) != float((dist.get_rank() - 1) % dist.get_world_size()):
            raise RuntimeError("received the wrong neighbour's buffer")
        dist.barrier()
        if dev.type == "cuda":
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                exchange(buf, out)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / iters
        else:
            t0 = time.perf_counter()
            for _ in range(iters):
                exchange(buf, out)
            ms = (time.perf_counter() - t0) * 1e3 / iters
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
        rows.append({"probe": "p2p_ring", "world": dist.get_world_size(), "mb": mb, "ms": ms,
                     "gbs_per_direction": (n * 4) / (ms * 1e-3) / 1e9, "backend": dist.get_backend()})
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", default="1,16,256")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    if not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    if torch.cuda.is_available():
        import os

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    try:
        rows = probe(tuple(float(x) for x in a.sizes_mb.split(",")), a.iters)
        if dist.get_rank() == 0:
            for r in rows:
                print(json.dumps(r), flush=True)
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
