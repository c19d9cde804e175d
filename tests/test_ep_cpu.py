"""Expert parallelism on CPU gloo ranks vs the single-process oracle (all experts local, dropless)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from marin_experiments_b200.ops import api
        from marin_experiments_b200.parallel.ep import moe_experts_ep

        torch.manual_seed(0)
        t, d, inter, e, k = 64, 32, 128, 8, 2
        e_loc = e // world
        xs = [torch.randn(t, d) for _ in range(world)]
        wr = torch.randn(e, d) / 4
        wgu = torch.randn(e, 2 * inter, d) / 8
        wdn = torch.randn(e, d, inter) / 8
        gouts = [torch.randn(t, d) for _ in range(world)]
        # oracle: all tokens of every rank through all experts, dropless
        oracle_grad_gu = torch.zeros_like(wgu)
        oracle_grad_d = torch.zeros_like(wdn)
        oracle_outs = []
        for rr in range(world):
            h = xs[rr].clone().requires_grad_(True)
            wg = wgu.clone().requires_grad_(True)
            wd = wdn.clone().requires_grad_(True)
            r = api.route(h, wr, torch.zeros(e), k, qb_count=8)
            y = api.moe_experts(h, r, wg, wd, capacity=None)
            y.backward(gouts[rr])
            oracle_grad_gu += wg.grad
            oracle_grad_d += wd.grad
            oracle_outs.append((y.detach(), h.grad.clone()))
        # EP
        h = xs[rank].clone().requires_grad_(True)
        lo, hi = rank * e_loc, (rank + 1) * e_loc
        wg = wgu[lo:hi].clone().requires_grad_(True)
        wd = wdn[lo:hi].clone().requires_grad_(True)
        r = api.route(h, wr, torch.zeros(e), k, qb_count=8)
        y = moe_experts_ep(h, r, wg, wd, api.capacity_for(t, k, 1, 1.0), dist.group.WORLD)
        y.backward(gouts[rank])
        ok = [
            torch.allclose(y.detach(), oracle_outs[rank][0], atol=1e-5, rtol=1e-4),
            torch.allclose(h.grad, oracle_outs[rank][1], atol=1e-5, rtol=1e-4),
            torch.allclose(wg.grad, oracle_grad_gu[lo:hi], atol=1e-5, rtol=1e-4),
            torch.allclose(wd.grad, oracle_grad_d[lo:hi], atol=1e-5, rtol=1e-4),
        ]
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_matches_oracle(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert all(results[r]), (r, results[r])
