"""Expert-parallel exchange kernels on their own: the four peer-memory exchanges of one MoE layer
(dispatch push, combine pull, combine-backward push, unpermute pull), each timed as the model runs
it (the kernel plus the flag wait for every peer) with CUDA events, max over ranks, against the
bytes that cross NVLink.

Routing is uniform random top-K over E experts (E / world per rank), capacity factor 1.25, so a
rank sends (world - 1) / world of its routed rows to other ranks.

Usage (one process per GPU):
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29531 -m marin_experiments_b200.benchmarks.ep_bench [--tokens 65536] [--iters 20]
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=65536)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--d", type=int, default=1536)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)

    from ..ops._ext import err_flag, ext
    from ..ops.cuda_fns import dispatch_plan
    from ..parallel import ep as EP

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    group = dist.new_group(list(range(world)))
    t, k, e, d = args.tokens, args.k, args.experts, args.d
    e_loc = e // world
    cap = int(math.ceil(t * k / e * 1.25 / 128) * 128)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    sel = torch.argsort(torch.rand(t, e, device=dev, generator=g), dim=1)[:, :k].int().contiguous()
    comb = torch.rand(t, k, device=dev, generator=g).float()
    keep = torch.ones(t, k, dtype=torch.bool, device=dev)
    slot, perm, wperm, counts = dispatch_plan(sel, keep, comb, e, cap)
    heap = EP._heap(group, dev, e, cap, d, 1)
    my = heap.my
    rows = e * cap
    off_x = heap.alloc("bench_x", rows * d * 2)
    off_cnt = heap.alloc("bench_cnt", e * 4)
    off_y = heap.alloc("bench_y", rows * d * 2)
    x = torch.randn(t, d, device=dev).bfloat16()
    out = torch.empty(t, d, dtype=torch.bfloat16, device=dev)
    y_local = torch.empty(rows, d, dtype=torch.bfloat16, device=dev)
    err = err_flag(dev)

    # rows this rank sends to (push) or reads from (pull) other ranks
    cnt = counts.clamp(max=cap).cpu()
    owner = torch.arange(e) // e_loc
    remote_rows = int(cnt[owner != my].sum())
    pad_rows = int(sum(((int(c) + 127) // 128) * 128 for c, o in zip(cnt.tolist(), owner.tolist()) if o != my))
    remote_bytes = remote_rows * d * 2

    def dispatch():
        ep = heap.next_epoch(EP._DISPATCH)
        ext().ep_dispatch_push(x, perm, counts, heap.peers, my, e_loc, cap, off_x, off_cnt, 0, EP._DISPATCH, ep,
                               heap.counter(EP._DISPATCH))
        ext().ep_wait(heap.peers, my, 0, EP._DISPATCH, ep, err)

    def combine():
        ey = heap.next_epoch(EP._Y)
        ext().ep_signal(heap.peers, my, 0, EP._Y, ey)
        ext().ep_wait(heap.peers, my, 0, EP._Y, ey, err)
        ext().ep_combine_pull(sel, slot, comb, None, out, y_local, heap.peers, my, e_loc, cap, off_y)

    def combine_bwd():
        edy = heap.next_epoch(EP._DY)
        ext().ep_combine_bwd_push(x, perm, wperm, counts, heap.peers, my, e_loc, cap, off_x, 0, EP._DY, edy,
                                  heap.counter(EP._DY))
        ext().ep_wait(heap.peers, my, 0, EP._DY, edy, err)

    def unpermute():
        exp_ = heap.next_epoch(EP._DXP)
        ext().ep_signal(heap.peers, my, 0, EP._DXP, exp_)
        ext().ep_wait(heap.peers, my, 0, EP._DXP, exp_, err)
        ext().ep_unpermute_pull(sel, slot, out, heap.peers, my, e_loc, cap, off_y)

    res = {}
    for name, fn, nbytes in (("dispatch_push", dispatch, pad_rows * d * 2), ("combine_pull", combine, remote_bytes),
                             ("combine_bwd_push", combine_bwd, pad_rows * d * 2),
                             ("unpermute_pull", unpermute, remote_bytes)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier(group=group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / args.iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=group)
        nb = torch.tensor([float(nbytes)], device=dev)
        dist.all_reduce(nb, op=dist.ReduceOp.MAX, group=group)
        res[name] = {"ms": ms.item(), "remote_MB": nb.item() / 1e6, "GBps": nb.item() / ms.item() / 1e6}
    if int(err.item()) != 0:
        raise RuntimeError(f"exchange wait timed out (error {int(err.item())})")
    if rank == 0:
        print(json.dumps({"ep_bench": {"world": world, "tokens": t, "k": k, "experts": e, "d": d, "cap": cap,
                                       "impl": os.environ.get("MXK_EP_XCHG", "v2"), "results": res}}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
