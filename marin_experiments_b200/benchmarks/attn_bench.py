"""Attention kernels: tcgen05 forward/backward vs the mma.sync ones and the library kernels on the
same box (cuDNN through torch's SDPA, flash_attn 2.x), causal, 16 heads x 96, 8 x 2048 tokens.

Usage: python -m marin_experiments_b200.benchmarks.attn_bench [--once] [--prof]

``--prof`` runs one forward with the kernel's phase counters on and prints their per-block means
(softmax warps: waiting for S, loads + row max, exponentials + P stores, rescale + release; MMA
thread: waiting for P, for K / V, for its own PV products).
"""

from __future__ import annotations

import json
import math

import torch


def fwd_phases(b=8, s=2048, h=16, hkv=16, hd=96) -> dict:
    """Per-block means of the tcgen05 forward's phase counters (SM clock cycles)."""
    from marin_experiments_b200.ops._ext import err_flag, ext

    t = b * s
    q = torch.randn(t, h, hd, device="cuda").bfloat16()
    k = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    v = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    o = torch.empty(t, h, hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(t, h, device="cuda")
    prof = torch.zeros(16, dtype=torch.int64, device="cuda")
    ext().flash_fwd_sm100(q, k, v, o, lse, None, b, s, 0, 1 / math.sqrt(hd), err_flag(q.device), None)
    ext().flash_fwd_sm100(q, k, v, o, lse, None, b, s, 0, 1 / math.sqrt(hd), err_flag(q.device), prof)
    torch.cuda.synchronize()
    p = prof.cpu().tolist()
    blocks = max(p[7], 1)
    ctas = (s + 255) // 256 * h * b
    res = {"softmax_wait_s": p[0] / blocks, "softmax_load_max": p[1] / blocks, "softmax_exp_store": p[2] / blocks,
           "softmax_rescale_release": p[3] / blocks, "mma_wait_p_per_cta": p[4] / ctas,
           "mma_wait_kv_per_cta": p[5] / ctas, "mma_wait_o_per_cta": p[6] / ctas, "rescales_per_block": p[8] / blocks}
    print(json.dumps({"fwd_phases": res}), flush=True)
    return res


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
    cases = [
        ("fwd_tcgen05", lambda: ext().flash_fwd_sm100(q, k, v, o, lse, None, b, s, 0, sc, err_flag(q.device), None), fl),
        ("fwd_mma_sync", lambda: ext().flash_fwd(q, k, v, o, lse, None, b, s, 0, sc), fl),
        ("bwd_mma_sync", lambda: ext().flash_bwd(q, k, v, o, lse, None, b, s, 0, sc, do, ds, dqa, dq, dk, dv, False),
         2.5 * fl),
        ("bwd_tcgen05", lambda: ext().flash_bwd_sm100(q, k, v, o, lse, None, b, s, 0, sc, do, ds, dqa, dq, dk, dv,
                                                      False, err_flag(q.device)), 2.5 * fl),
    ]
    cases += _library_cases(b, s, h, hkv, hd, fl)
    for name, fn, f in cases:
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


def _library_cases(b, s, h, hkv, hd, fl):
    """cuDNN attention (torch SDPA restricted to the cuDNN backend) and flash_attn, forward and
    forward+backward minus forward, on the same shape; skipped where the library is missing."""
    out = []
    q = torch.randn(b, h, s, hd, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(b, hkv, s, hd, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(b, hkv, s, hd, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    do = torch.randn(b, h, s, hd, device="cuda", dtype=torch.bfloat16)
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        import torch.nn.functional as F

        def cudnn_fwd():
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                return F.scaled_dot_product_attention(q, k, v, is_causal=True)

        cudnn_fwd()
        o = cudnn_fwd()

        def cudnn_bwd():
            torch.autograd.grad(o, (q, k, v), do, retain_graph=True)

        cudnn_bwd()
        out += [("fwd_cudnn", cudnn_fwd, fl), ("bwd_cudnn", cudnn_bwd, 2.5 * fl)]
    except Exception as e:  # backend not available for this shape / build
        print(json.dumps({"cudnn": f"unavailable: {type(e).__name__}: {e}"[:200]}), flush=True)
    try:
        from flash_attn import flash_attn_func

        qf, kf, vf = (t.detach().transpose(1, 2).contiguous().requires_grad_(True) for t in (q, k, v))
        dof = do.transpose(1, 2).contiguous()

        def fa_fwd():
            return flash_attn_func(qf, kf, vf, causal=True)

        of = fa_fwd()

        def fa_bwd():
            torch.autograd.grad(of, (qf, kf, vf), dof, retain_graph=True)

        fa_bwd()
        out += [("fwd_flash_attn", fa_fwd, fl), ("bwd_flash_attn", fa_bwd, 2.5 * fl)]
    except Exception as e:
        print(json.dumps({"flash_attn": f"unavailable: {type(e).__name__}: {e}"[:200]}), flush=True)
    return out


if __name__ == "__main__":
    import sys

    if "--prof" in sys.argv:
        fwd_phases()
    else:
        run(once="--once" in sys.argv)
