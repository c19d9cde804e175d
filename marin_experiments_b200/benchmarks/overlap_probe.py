"""Compute / communication overlap probe (megagpt-speedrun/pp_overlap_probe.py:55-484,
grug-moe-pp/overlap_probe.py): time a GEMM loop alone, an NCCL all-reduce loop alone, and both on
separate CUDA streams at once; overlap factor = (t_gemm + t_comm) / t_both (2.0 = perfect).

Run: ``python -m torch.distributed.run --nproc-per-node N -m marin_experiments_b200.benchmarks.overlap_probe``
(rank 0 prints one JSON line). Device-timed with CUDA events, max over ranks.
"""

from __future__ import annotations

import datetime
import json
import os

import torch
import torch.distributed as dist


def _timed(fn, stream=None) -> float:
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def main(m: int = 8192, n: int = 8192, k: int = 8192, comm_mb: int = 512, iters: int = 10):
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    rank = dist.get_rank()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    from marin_experiments_b200.ops import gemm as G

    a = torch.randn(m, k, device="cuda").bfloat16()
    b = torch.randn(n, k, device="cuda").bfloat16()
    c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    buf = torch.randn(comm_mb * (1 << 20) // 4, device="cuda")
    s_comm = torch.cuda.Stream()

    def gemms():
        for _ in range(iters):
            G.gemm(a, b, c, M=m, N=n, K=k)

    def comms():
        with torch.cuda.stream(s_comm):
            for _ in range(iters):
                dist.all_reduce(buf)
        torch.cuda.current_stream().wait_stream(s_comm)

    def both():
        s_comm.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_comm):
            for _ in range(iters):
                dist.all_reduce(buf)
        gemms()
        torch.cuda.current_stream().wait_stream(s_comm)

    for f in (gemms, comms, both):
        f()
    t = torch.tensor([_timed(gemms), _timed(comms), _timed(both)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tg, tc, tb = (float(x) for x in t)
    if rank == 0:
        print(json.dumps({"gemm_ms": tg, "allreduce_ms": tc, "both_ms": tb, "overlap_factor": (tg + tc) / tb,
                          "gemm_tflops": 2 * m * n * k * iters / tg / 1e9,
                          "allreduce_busbw_gbs": 2 * (dist.get_world_size() - 1) / dist.get_world_size()
                          * buf.numel() * 4 * iters / tc / 1e6, "ranks": dist.get_world_size()}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
