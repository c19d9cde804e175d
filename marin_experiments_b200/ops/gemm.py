"""Python front end of the sm_100a tcgen05 GEMM (``csrc/gemm_sm100.cuh``).

Conventions: ``C = A' @ B'^T`` where ``A'`` is ``[M, K]`` and ``B'`` is ``[N, K]``. A K-major
operand is passed as stored (``[rows, K]``); an MN-major operand is passed as its stored
``[K, rows]`` tensor with ``*_mn=True``. Linear layers keep weights ``[out, in]`` so that

* forward  ``y  = x @ W^T``      -> A = x (K-major),   B = W (K-major)
* input    ``dx = dy @ W``       -> A = dy (K-major),  B = W (MN-major)
* weight   ``dW = dy^T @ x``     -> A = dy (MN-major), B = x (MN-major)
"""

from __future__ import annotations

import contextlib

import torch

from ._ext import err_flag, ext

EPI = {"store": 0, "swiglu": 1, "resid": 2, "gate_mul": 3, "silu": 4, "rowscale": 5, "ce": 6, "act": 7,
       "swiglu_bwd": 8}
ACT = {"silu": 0, "relu": 1, "gelu": 2}


def _pick_bn(n: int, epi: str, b_mn: bool, a_mn: bool) -> int:
    if epi in ("swiglu", "ce", "swiglu_bwd"):
        return 256
    if epi == "silu":
        return 128
    if n >= 512:
        return 256
    if n >= 128:
        return 128
    return 64


def gemm(a, b, c, *, a_mn=False, b_mn=False, G=1, M=None, N=None, K=None, counts=None, ragged=0,
         a_grp=0, b_grp=0, c_grp=0, epi="store", bn=None, accum=False, alpha=1.0, c2=None, r=None,
         row_scale=None, act="silu", b_mod=0, c_mod=0, peer=None):
    """``peer = (maps, epl, my, cap)``: store group g's rows into rank g // epl's buffer instead of
    ``c`` (see ``PeerStore``)."""
    if bn is None:
        bn = _pick_bn(N, epi, b_mn, a_mn)
    maps, epl, my, pcap = peer if peer is not None else (None, 0, 0, 0)
    ext().gemm(a, a_mn, b, b_mn, c, G, M, N, K, counts, ragged, a_grp, b_grp, c_grp, EPI[epi], bn, int(accum),
               float(alpha), c2, r, row_scale, ACT[act], err_flag(a.device), b_mod, c_mod, maps, epl, my, pcap)
    return c


def linear(x, w, *, out=None, epi="store", **kw):
    """``x [M, K] @ w[N, K]^T`` -> ``[M, N]`` bf16 (or into ``out``)."""
    m, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    return gemm(x, w, out, M=m, N=n, K=k, epi=epi, **kw)


def linear_dx(dy, w, *, out=None, accum=False, swiglu_h=None):
    """``dy [M, N] @ w [N, K]`` -> ``[M, K]``. With ``swiglu_h`` (the SwiGLU pre-activations
    ``[M, 2K]``, blocked gate/up) the epilogue turns the activation gradient into the gate/up
    gradients ``[M, 2K]`` (SiLU gate)."""
    m, n = dy.shape
    k = w.shape[1]
    if swiglu_h is not None:
        if out is None:
            out = torch.empty(m, 2 * k, dtype=torch.bfloat16, device=dy.device)
        return gemm(dy, w, out, b_mn=True, M=m, N=k, K=n, epi="swiglu_bwd", r=swiglu_h)
    if out is None:
        out = torch.empty(m, k, dtype=torch.bfloat16, device=dy.device)
    return gemm(dy, w, out, b_mn=True, M=m, N=k, K=n, accum=accum)


class _WeightGradQueue:
    # Process-wide, not thread-local: autograd runs CUDA backward functions on its own device
    # threads, which must see the queue the caller installed. One backward at a time per process.
    queue = None


_WGQ = _WeightGradQueue()


@contextlib.contextmanager
def defer_weight_grads(queue: list):
    """Within this context, backward passes queue their weight-gradient GEMMs (the ones that
    accumulate into a parameter's ``main_grad``) on ``queue`` instead of launching them, so a
    zero-bubble pipeline schedule can run the input-gradient pass (B) now and the weight-gradient
    pass (W) later: ``run_weight_grads(queue)``."""
    prev = _WGQ.queue
    _WGQ.queue = queue
    try:
        yield queue
    finally:
        _WGQ.queue = prev


def run_weight_grads(queue: list) -> None:
    while queue:
        queue.pop(0)()


def weight_grad(fn) -> None:
    """Run ``fn`` (a weight-gradient accumulation) now, or queue it inside ``defer_weight_grads``."""
    if _WGQ.queue is not None:
        _WGQ.queue.append(fn)
    else:
        fn()


def linear_dw(dy, x, *, out=None, accum=False, alpha=1.0):
    """``dy [T, N]^T @ x [T, K]`` -> ``[N, K]`` (fp32 when accumulating into a main grad)."""
    t, n = dy.shape
    k = x.shape[1]
    if out is None:
        out = torch.empty(n, k, dtype=torch.float32, device=dy.device)
    if accum:
        weight_grad(lambda: gemm(dy, x, out, a_mn=True, b_mn=True, M=n, N=k, K=t, accum=accum, alpha=alpha))
        return out
    return gemm(dy, x, out, a_mn=True, b_mn=True, M=n, N=k, K=t, accum=accum, alpha=alpha)


class PeerStore:
    """Destination of a grouped GEMM whose output rows belong to other GPUs: group ``g = s * epl + e``
    (source rank s, local expert e) is written into rank s's ``[E][cap][N]`` buffer at rows
    ``(my * epl + e) * cap + ...`` by the GEMM's own epilogue (TMA stores into peer memory), so the
    transfer overlaps the math tile by tile. ``maps`` is the device array of per-rank tensor maps
    from ``ext().peer_store_maps``."""

    def __init__(self, maps: torch.Tensor, epl: int, my: int, cap: int):
        self.maps, self.epl, self.my, self.cap = maps, epl, my, cap

    def args(self):
        return (self.maps, self.epl, self.my, self.cap)


def grouped_linear(x, w, counts, *, out=None, epi="store", c2=None, n_w=None, **kw):
    """Per-group ``x[g] @ w[g % n_w]^T`` over a capacity layout.

    x: ``[G*C, K]`` (group g owns rows ``[g*C, (g+1)*C)``, only the first ``counts[g]`` valid),
    w: ``[n_w*N, K]`` -> out ``[G*C, N]``; tiles past ``counts[g]`` rows are skipped. ``n_w < G`` lets
    several activation groups (one per source rank) share an expert's weights."""
    g = counts.numel()
    n_w = n_w or g
    cap = x.shape[0] // g
    n = w.shape[0] // n_w
    k = x.shape[1]
    if out is None:
        out = torch.empty(x.shape[0], n, dtype=torch.bfloat16, device=x.device)
    peer = kw.pop("peer", None)
    if peer is not None:
        kw["peer"] = peer.args()
    return gemm(x, w, out, G=g, M=cap, N=n, K=k, counts=counts, ragged=1, a_grp=cap, b_grp=n, c_grp=cap,
                epi=epi, c2=c2, b_mod=0 if n_w == g else n_w, **kw)


def grouped_linear_dx(dy, w, counts, *, out=None, n_w=None, swiglu_h=None, peer=None):
    """Per-group ``dy[g] [C, N] @ w[g % n_w] [N, K]`` -> ``[G*C, K]``. With ``swiglu_h`` (the SwiGLU
    pre-activations ``[G*C, 2K]``, blocked gate/up rows) the product is the activation gradient and
    the epilogue writes the gate/up gradients ``[G*C, 2K]`` instead (SiLU gate)."""
    g = counts.numel()
    n_w = n_w or g
    cap = dy.shape[0] // g
    n = w.shape[0] // n_w
    k = w.shape[1]
    if out is None:
        cols = 2 * k if swiglu_h is not None else k
        out = torch.empty(dy.shape[0], cols, dtype=torch.bfloat16, device=dy.device)
    extra = {} if swiglu_h is None else {"epi": "swiglu_bwd", "r": swiglu_h}
    if peer is not None:
        extra["peer"] = peer.args()
    return gemm(dy, w, out, b_mn=True, G=g, M=cap, N=k, K=n, counts=counts, ragged=1, a_grp=cap, b_grp=n,
                c_grp=cap, b_mod=0 if n_w == g else n_w, **extra)


def grouped_linear_dw(dy, x, counts, *, out, accum=True, alpha=1.0, n_w=None):
    """Per-group ``dy[g]^T @ x[g]`` contracting over the first ``counts[g]`` rows (rounded up to
    64; rows past the count must be zero), accumulated into ``out [n_w*N, K]`` fp32 at weight group
    ``g % n_w`` (with atomics when several groups share a weight group)."""
    g = counts.numel()
    n_w = n_w or g
    cap = dy.shape[0] // g
    n = dy.shape[1]
    k = x.shape[1]
    shared = n_w != g
    weight_grad(lambda: gemm(dy, x, out, a_mn=True, b_mn=True, G=g, M=n, N=k, K=cap, counts=counts, ragged=2,
                             a_grp=cap, b_grp=cap, c_grp=n, accum=(2 if shared else accum), alpha=alpha,
                             c_mod=n_w if shared else 0))
    return out
