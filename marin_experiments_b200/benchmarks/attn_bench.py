"""Attention kernels: tcgen05 forward/backward vs the mma.sync ones, causal, 16 heads x 96.

Usage: python -m marin_experiments_b200.benchmarks.attn_bench
"""

from __future__ import annotations

import json
import math

import torch


def run(b=8, s=2048, h=16, hkv=16, hd=96, iters=10, once=False):
    """Time the tcgen05 and mma.sync kernels (CUDA events, ``iters`` back-to-back launches after
    3 warm-ups). ``once``: one tcgen05 forward and one backward, untimed (a launch list for ncu)."""
    from marin_experiments_b200.ops._ext import err_flag, ext

    t = b * s
    q = torch.randn(t, h, hd, device="cuda").bfloat16()
    k = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    v = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    o = torch.empty(t, h, hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(t, h, device="cuda")
    do = torch.randn_like(o)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.zeros_like(v)
    dqa = torch.empty(t, h, hd, device="cuda")
    ds = torch.empty(t, h, device="cuda")
    sc = 1 / math.sqrt(hd)
    fl = 4.0 * b * h * hd * s * s / 2  # causal forward FLOPs
    res = {}
    if once:
        ext().flash_fwd_sm100(q, k, v, o, lse, None, b, s, 0, sc, err_flag(q.device), None)
        ext().flash_bwd_sm100(q, k, v, o, lse, None, b, s, 0, sc, do, ds, dqa, dq, dk, dv, False, err_flag(q.device))
        torch.cuda.synchronize()
        return res
    for name, fn, f in [
        ("fwd_tcgen05", lambda: ext().flash_fwd_sm100(q, k, v, o, lse, None, b, s, 0, sc, err_flag(q.device), None), fl),
        ("fwd_mma_sync", lambda: ext().flash_fwd(q, k, v, o, lse, None, b, s, 0, sc), fl),
        ("bwd_mma_sync", lambda: ext().flash_bwd(q, k, v, o, lse, None, b, s, 0, sc, do, ds, dqa, dq, dk, dv, False),
         2.5 * fl),
        ("bwd_tcgen05", lambda: ext().flash_bwd_sm100(q, k, v, o, lse, None, b, s, 0, sc, do, ds, dqa, dq, dk, dv,
                                                      False, err_flag(q.device)), 2.5 * fl),
    ]:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / iters
        res[name] = {"ms": ms, "tflops": f / ms / 1e9}
        print(json.dumps({name: res[name]}), flush=True)
    return res


if __name__ == "__main__":
    import sys

    run(once="--once" in sys.argv)
