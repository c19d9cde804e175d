"""Expert-parallel MoE on 2+ GPUs (NCCL) vs each rank's own all-experts computation."""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from marin_experiments_b200.ops import api
        from marin_experiments_b200.parallel.ep import moe_experts_ep

        def rel(a, b):
            return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()

        torch.manual_seed(0)
        t, d, inter, e, k = 1024, 256, 256, 16, 2
        e_loc = e // world
        xs = [torch.randn(t, d).bfloat16() for _ in range(world)]
        wr = (torch.randn(e, d) / 8).bfloat16()
        wgu = (torch.randn(e, 2 * inter, d) / 16).bfloat16()
        wdn = (torch.randn(e, d, inter) / 16).bfloat16()
        gout = torch.randn(t, d).bfloat16()
        dev = torch.device("cuda", rank)

        def param(x):
            p = x.to(dev).requires_grad_(True)
            p.main_grad = torch.zeros(x.shape, dtype=torch.float32, device=dev)
            return p

        cap = api.capacity_for(t, k, e, 4.0)  # generous: no drops
        # EP
        h = xs[rank].to(dev).requires_grad_(True)
        lo, hi = rank * e_loc, (rank + 1) * e_loc
        wg, wd = param(wgu[lo:hi]), param(wdn[lo:hi])
        r = api.route(h, param(wr), torch.zeros(e, device=dev), k, qb_count=64)
        y = moe_experts_ep(h, r, wg, wd, cap, dist.group.WORLD)
        y.backward(gout.to(dev))
        # reference on this GPU: all ranks' tokens through all experts
        full_gu, full_d = param(wgu), param(wdn)
        hr = None
        for rr in range(world):
            hh = xs[rr].to(dev).requires_grad_(True)
            rt = api.route(hh, param(wr), torch.zeros(e, device=dev), k, qb_count=64)
            yy = api.moe_experts(hh, rt, full_gu, full_d, capacity=api.capacity_for(t, k, e, 4.0))
            yy.backward(gout.to(dev))
            if rr == rank:
                y_ref, hr = yy.detach(), hh.grad
        res = [rel(y, y_ref), rel(h.grad, hr), rel(wg.main_grad, full_gu.main_grad[lo:hi]),
               rel(wd.main_grad, full_d.main_grad[lo:hi])]
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_gpu_matches_single_gpu():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert all(v < 2e-2 for v in results[r]), (r, results[r])
