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

    world = min(torch.cuda.device_count(), 8)
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


def _worker_impls(rank, world, port, q):
    """Peer-memory exchange vs NCCL all-to-all on the same inputs: 2 layers x 3 iterations of
    forward + backward (exercises the per-layer buffers, shared buffers and epochs)."""
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from marin_experiments_b200.ops import api
        from marin_experiments_b200.ops._ext import check_kernel_errors
        from marin_experiments_b200.parallel import ep

        dev = torch.device("cuda", rank)
        t, d, inter, e, k = 2048, 256, 256, 8, 2  # capacity 1024: two 512-slot dispatch chunks
        e_loc = e // world
        lo, hi = rank * e_loc, (rank + 1) * e_loc

        def param(x):
            p = x.to(dev).requires_grad_(True)
            p.main_grad = torch.zeros(x.shape, dtype=torch.float32, device=dev)
            return p

        g = torch.Generator().manual_seed(3)
        layers = [((torch.randn(e, d, generator=g) / 8).bfloat16(), (torch.randn(e, 2 * inter, d, generator=g) / 16).bfloat16(),
                   (torch.randn(e, d, inter, generator=g) / 16).bfloat16()) for _ in range(2)]
        gx = torch.Generator().manual_seed(100 + rank)
        xs = [torch.randn(t, d, generator=gx).bfloat16() for _ in range(3)]
        gouts = [torch.randn(t, d, generator=gx).bfloat16() for _ in range(3)]
        res = {}
        from marin_experiments_b200.ops._ext import ext

        variants = [("nccl", "store", "1"), ("peer", "pull", "1"), ("peer", "store", "1")]
        if "s_lo" in (ext().ep_dispatch_push.__doc__ or ""):  # a build with the chunked dispatch
            variants.append(("peer", "pull", "2"))
        for impl, ret, chunks in variants:
            os.environ["MXK_EP_IMPL"] = impl
            os.environ["MXK_EP_RETURN"] = ret  # store: rows return inside the GEMM epilogues
            os.environ["MXK_EP_CHUNKS"] = chunks  # 2: dispatch in two chunks beside the first GEMM
            impl = impl if impl == "nccl" else f"peer-{ret}" + ("-chunked" if chunks == "2" else "")
            params = [(param(wr), param(wgu[lo:hi]), param(wdn[lo:hi])) for wr, wgu, wdn in layers]
            outs, grads = [], []
            for it in range(3):
                h0 = xs[it].to(dev).requires_grad_(True)
                h = h0
                for li, (wr, wg, wd) in enumerate(params):
                    r = api.route(h, wr, torch.zeros(e, device=dev), k, qb_count=32)
                    h = ep.moe_experts_ep(h, r, wg, wd, api.capacity_for(t, k, e, 2.0), dist.group.WORLD, residual=h,
                                          layer=li, n_layers=2)
                h.backward(gouts[it].to(dev))
                outs.append(h.detach().float().cpu())
                grads.append(h0.grad.float().cpu())
            torch.cuda.synchronize()
            check_kernel_errors()
            res[impl] = (outs, grads, [p[1].main_grad.cpu() for p in params], [p[2].main_grad.cpu() for p in params])

        def rel(a, b):
            return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()

        errs = []
        for name in [n for n in ("peer-pull", "peer-store", "peer-pull-chunked") if n in res]:
            got, want = res[name], res["nccl"]
            errs += [rel(a, b) for a, b in zip(got[0] + got[1] + got[2] + got[3],
                                               want[0] + want[1] + want[2] + want[3])]
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_peer_exchange_matches_nccl():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_impls, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert all(v < 1e-2 for v in results[r]), (r, results[r])


def _worker_overlap(rank, world, port, q):
    """Shared expert on a side stream during the exchange vs the sequential composition: 4 forward +
    backward passes of one MoE layer each, alternating between two layers' buffers; outputs, input
    gradients and the shared and routed experts' weight gradients (read right after backward, on the
    training stream). One layer per pass keeps the routing identical in both modes: the two modes
    add the shared and routed outputs to the residual in a different order, and a second layer's
    top-k would flip for near-tied tokens on that rounding difference."""
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["MXK_EP_IMPL"] = "peer"
    os.environ["MXK_EP_OVERLAP"] = "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from marin_experiments_b200.ops import api
        from marin_experiments_b200.ops._ext import check_kernel_errors
        from marin_experiments_b200.parallel import ep

        dev = torch.device("cuda", rank)
        t, d, inter, e, k, si = 1024, 256, 256, 8, 2, 512
        e_loc = e // world
        lo, hi = rank * e_loc, (rank + 1) * e_loc

        def param(x):
            p = x.to(dev).requires_grad_(True)
            p.main_grad = torch.zeros(x.shape, dtype=torch.float32, device=dev)
            return p

        g = torch.Generator().manual_seed(5)
        layers = [((torch.randn(e, d, generator=g) / 8).bfloat16(),
                   (torch.randn(e, 2 * inter, d, generator=g) / 16).bfloat16(),
                   (torch.randn(e, d, inter, generator=g) / 16).bfloat16(),
                   (torch.randn(2 * si, d, generator=g) / 16).bfloat16(),
                   (torch.randn(d, si, generator=g) / 16).bfloat16()) for _ in range(2)]
        gx = torch.Generator().manual_seed(200 + rank)
        xs = [torch.randn(t, d, generator=gx).bfloat16() for _ in range(4)]
        gouts = [torch.randn(t, d, generator=gx).bfloat16() for _ in range(4)]
        res = {}
        for mode in ("sequential", "overlap"):
            params = [(param(wr), param(wgu[lo:hi]), param(wdn[lo:hi]), param(sgu), param(sdn))
                      for wr, wgu, wdn, sgu, sdn in layers]
            outs, grads = [], []
            for it in range(4):
                h0 = xs[it].to(dev).requires_grad_(True)
                h = h0
                for li in (it % 2,):
                    wr, wg, wd, sg, sd = params[li]
                    r = api.route(h, wr, torch.zeros(e, device=dev), k, qb_count=32)
                    cap = api.capacity_for(t, k, e, 2.0)
                    if mode == "sequential":
                        base = api.dense_mlp(h, sg, sd, glu=True, act="silu", residual=h)
                        h = ep.moe_experts_ep(h, r, wg, wd, cap, dist.group.WORLD, residual=base, layer=li,
                                              n_layers=2)
                    else:
                        assert ep.overlap_shared_enabled(h, dist.group.WORLD)
                        hh, rr = h, r
                        h, _ = ep.with_shared_overlap(
                            hh, lambda z, sg=sg, sd=sd: api.dense_mlp(z, sg, sd, glu=True, act="silu"),
                            lambda hh=hh, rr=rr, wg=wg, wd=wd, li=li: (
                                ep.moe_experts_ep(hh, rr, wg, wd, cap, dist.group.WORLD, residual=hh, layer=li,
                                                  n_layers=2), None))
                h.backward(gouts[it].to(dev))
                outs.append(h.detach().float().cpu())
                grads.append(h0.grad.float().cpu())
            mg = [[p[j].main_grad.cpu() for p in params] for j in (1, 2, 3, 4)]
            torch.cuda.synchronize()
            check_kernel_errors()
            res[mode] = (outs, grads, *mg)

        def rel(a, b):
            return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()

        errs = [rel(a, b) for ga, gb in zip(res["overlap"], res["sequential"]) for a, b in zip(ga, gb)]
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_shared_expert_overlap_matches_sequential():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_overlap, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert all(v < 1e-2 for v in results[r]), (r, results[r])
