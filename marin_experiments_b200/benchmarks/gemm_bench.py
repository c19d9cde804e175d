"""Throughput of the sm_100a GEMM against cuBLAS (torch.matmul) on the model's shapes.

Timing: CUDA events on the launching stream after warm-up; an L2-sized buffer is rewritten
between timed launches so every launch reads its operands from HBM.
Usage: python -m marin_experiments_b200.benchmarks.gemm_bench [--json out.json]
"""

from __future__ import annotations

import argparse
import json

import torch

from marin_experiments_b200.ops import gemm as G

SHAPES = [
    # (name, M, N, K, mode)
    ("square8192", 8192, 8192, 8192, "fwd"),
    ("qkv_fwd", 16384, 4608, 1536, "fwd"),
    ("o_fwd", 16384, 1536, 1536, "fwd"),
    ("shared_gateup_fwd", 16384, 6144, 1536, "fwd"),
    ("shared_down_fwd", 16384, 1536, 3072, "fwd"),
    ("lm_head_fwd", 16384, 128256, 1536, "fwd"),
    ("o_dx", 16384, 1536, 1536, "dx"),
    ("o_dw", 16384, 1536, 1536, "dw"),
    ("lm_head_dw", 16384, 128256, 1536, "dw"),
    # GatedNorm (rank 128) and residual-epilogue shapes
    ("gatednorm_up_gate_mul", 16384, 1536, 128, "gate_mul"),
    ("gatednorm_down_silu", 16384, 128, 1536, "silu"),
    ("o_fwd_resid", 16384, 1536, 1536, "resid"),
    ("gatednorm_dw_up", 16384, 1536, 128, "dw"),
    # grouped expert weight gradients (64 experts, ragged K = 1024 tokens each, fp32 accumulate)
    ("expert_gateup_dw", 1536, 1536, 1024, "gdw"),
    ("expert_down_dw", 1536, 768, 1024, "gdw"),
    # expert forward / input-gradient GEMMs as the MoE layer runs them: 64 experts, 1280-row capacity
    # slots holding 1024 routed tokens each; M = tokens per expert, N = out, K = in
    ("expert_gateup_fwd_swiglu", 1024, 1536, 1536, "gfwd"),
    ("expert_down_fwd", 1024, 1536, 768, "gfwd"),
    ("expert_down_dx_swiglu_bwd", 1024, 1536, 768, "gdx"),
    ("expert_gateup_dx", 1024, 1536, 1536, "gdx"),
    ("shared_gateup_dw", 16384, 6144, 1536, "dw"),
    ("qkv_dw", 16384, 2304, 1536, "dw"),
]


def _time(fn, flush, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    return ts[len(ts) // 2]


def run(shapes=SHAPES, once: bool = False):
    """Time every shape against torch.matmul (median of 10, L2 flushed). ``once``: launch our GEMM
    a single time per shape and time nothing (a small, fixed launch list for ncu captures)."""
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    rows = []
    for name, m, n, k, mode in shapes:
        if mode == "fwd":
            a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            b = torch.randn(n, k, device="cuda").to(torch.bfloat16)
            c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.linear(a, b, out=c)
            ref = lambda: torch.matmul(a, b.t(), out=c)
        elif mode == "dx":
            a = torch.randn(m, n, device="cuda").to(torch.bfloat16)  # dy
            b = torch.randn(n, k, device="cuda").to(torch.bfloat16)  # w
            c = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.linear_dx(a, b, out=c)
            ref = lambda: torch.matmul(a, b, out=c)
        elif mode in ("gate_mul", "resid"):
            a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            b = torch.randn(n, k, device="cuda").to(torch.bfloat16)
            r = torch.randn(m, n, device="cuda").to(torch.bfloat16)
            c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.gemm(a, b, c, M=m, N=n, K=k, epi=mode, r=r)
            ref = (lambda: torch.mul(r, torch.sigmoid(torch.matmul(a, b.t())), out=c)) if mode == "gate_mul" else \
                (lambda: torch.add(r, torch.matmul(a, b.t()), out=c))
        elif mode == "silu":
            a = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            b = torch.randn(n, k, device="cuda").to(torch.bfloat16)
            c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            h = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.gemm(a, b, c, M=m, N=n, K=k, epi="silu", c2=h)
            ref = lambda: torch.nn.functional.silu(torch.matmul(a, b.t(), out=h), inplace=False)
        elif mode == "gdw":  # per expert: dy [cap, m]^T x [cap, n] -> [m, n] fp32, K = k tokens
            ge, cap = 64, 1280
            cnt = torch.full((ge,), k, dtype=torch.int32, device="cuda")
            a = torch.randn(ge * cap, m, device="cuda").to(torch.bfloat16)
            b = torch.randn(ge * cap, n, device="cuda").to(torch.bfloat16)
            c = torch.zeros(ge * m, n, device="cuda", dtype=torch.float32)
            a3, b3 = a.view(ge, cap, m)[:, :k], b.view(ge, cap, n)[:, :k]
            cb = torch.empty(ge, m, n, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.grouped_linear_dw(a, b, cnt, out=c)
            ref = lambda: torch.bmm(a3.transpose(1, 2), b3, out=cb)
            flops_mult = ge
        elif mode == "gfwd":  # per expert: x [tokens, k] @ w[n, k]^T; gate/up rows get the SwiGLU epilogue
            ge, cap = 64, 1280
            cnt = torch.full((ge,), m, dtype=torch.int32, device="cuda")
            a = torch.randn(ge * cap, k, device="cuda").to(torch.bfloat16)
            b = torch.randn(ge * n, k, device="cuda").to(torch.bfloat16)
            c = torch.empty(ge * cap, n, device="cuda", dtype=torch.bfloat16)
            sw = name.endswith("swiglu")
            act = torch.empty(ge * cap, n // 2, device="cuda", dtype=torch.bfloat16) if sw else None
            a3, b3 = a.view(ge, cap, k)[:, :m], b.view(ge, n, k)
            cb = torch.empty(ge, m, n, device="cuda", dtype=torch.bfloat16)
            mine = (lambda: G.grouped_linear(a, b, cnt, out=c, epi="swiglu", c2=act)) if sw else \
                (lambda: G.grouped_linear(a, b, cnt, out=c))
            ref = lambda: torch.bmm(a3, b3.transpose(1, 2), out=cb)
            flops_mult = ge
        elif mode == "gdx":  # per expert: dy [tokens, n] @ w[n, k]; swiglu_bwd writes gate/up grads
            ge, cap = 64, 1280
            cnt = torch.full((ge,), m, dtype=torch.int32, device="cuda")
            a = torch.randn(ge * cap, n, device="cuda").to(torch.bfloat16)
            b = torch.randn(ge * n, k, device="cuda").to(torch.bfloat16)
            sw = name.endswith("swiglu_bwd")
            hh = torch.randn(ge * cap, 2 * k, device="cuda").to(torch.bfloat16) if sw else None
            a3, b3 = a.view(ge, cap, n)[:, :m], b.view(ge, n, k)
            cb = torch.empty(ge, m, k, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.grouped_linear_dx(a, b, cnt, swiglu_h=hh)
            ref = lambda: torch.bmm(a3, b3, out=cb)
            flops_mult = ge
            c = None
        else:  # dw: dy [m, n], x [m, k] -> [n, k] fp32 accumulate
            a = torch.randn(m, n, device="cuda").to(torch.bfloat16)
            b = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            c = torch.zeros(n, k, device="cuda", dtype=torch.float32)
            cb = torch.empty(n, k, device="cuda", dtype=torch.bfloat16)
            mine = lambda: G.linear_dw(a, b, out=c, accum=True)
            ref = lambda: torch.matmul(a.t(), b, out=cb)
        flops = 2.0 * m * n * k * (flops_mult if mode in ("gdw", "gfwd", "gdx") else 1)
        if once:
            mine()
            torch.cuda.synchronize()
            continue
        t_mine = _time(mine, flush)
        t_ref = _time(ref, flush)
        rows.append({"name": name, "M": m, "N": n, "K": k, "mode": mode, "ms": t_mine, "cublas_ms": t_ref,
                     "tflops": flops / t_mine / 1e9, "cublas_tflops": flops / t_ref / 1e9})
        print(json.dumps(rows[-1]), flush=True)
        del a, b, c
    return rows


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--only", default=None, help="comma-separated shape names")
    ap.add_argument("--once", action="store_true", help="one untimed launch per shape (for ncu)")
    args = ap.parse_args()
    shapes = SHAPES if args.only is None else [s for s in SHAPES if s[0] in args.only.split(",")]
    rows = run(shapes, once=args.once)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)
