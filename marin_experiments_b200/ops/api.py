"""Public op API used by the models.

Every op takes flattened token tensors (``[T, ...]`` with ``T = B * S``). On CUDA tensors the op
runs the sm_100a kernels through hand-written autograd Functions (``ops.cuda_fns``), which
accumulate weight gradients straight into each parameter's fp32 ``main_grad``; if the compiled
extension is missing this raises. On CPU tensors the op evaluates the fp32 oracle
(``ops.reference``) under torch autograd -- the same definitions the kernels are tested against.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import reference as R
from .layout import split_gate_up


def _cuda():
    from . import cuda_fns

    return cuda_fns


# ---------------------------------------------------------------------------------- embedding


def embed(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    if ids.is_cuda:
        return _cuda().embed(ids, table)
    return F.embedding(ids, table)


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w^T`` (+ residual)."""
    if x.is_cuda:
        return _cuda().linear(x, w, residual)
    y = x @ w.t().to(x.dtype)
    return y if residual is None else residual + y


# ------------------------------------------------------------------------------ norms


def rms_gated_norm(x, w_rms, eps: float, w_down=None, w_up=None):
    """RMSNorm followed (optionally) by GatedNorm (megagpt-speedrun/model.py:288-328)."""
    if x.is_cuda:
        return _cuda().rms_gated_norm(x, w_rms, eps, w_down, w_up)
    y = R.rms_norm(x, w_rms, eps)
    if w_down is not None:
        y = R.gated_norm(y, w_down, w_up)
    return y


def rms_gated_norm_res(x, w_rms, eps: float, w_down=None, w_up=None):
    """``(norm(x), residual)``: the normalised input and the tensor to use as the block's residual
    stream (on CUDA an alias of ``x`` whose gradient is summed inside the norm's backward kernel)."""
    if x.is_cuda:
        return _cuda().rms_gated_norm(x, w_rms, eps, w_down, w_up, passthrough=True)
    return rms_gated_norm(x, w_rms, eps, w_down, w_up), x


# -------------------------------------------------------------------------------- attention


class AttnShape:
    """Static description of one attention call."""

    def __init__(self, batch, seq, heads, kv_heads, head_dim, window=0, qk_mult=1.0, qk_norm=True,
                 xsa=True, head_gate=True, rope_theta=10000.0, llama3=None):
        self.batch, self.seq, self.heads, self.kv_heads, self.head_dim = batch, seq, heads, kv_heads, head_dim
        self.window, self.qk_mult, self.qk_norm = window, qk_mult, qk_norm
        self.xsa, self.head_gate = xsa, head_gate
        self.rope_theta, self.llama3 = rope_theta, llama3

    @property
    def q_cols(self):
        return self.heads * self.head_dim

    @property
    def kv_cols(self):
        return self.kv_heads * self.head_dim


_ROPE_CACHE: dict = {}


def rope_tables(seq, head_dim, theta, device, llama3=None):
    key = (seq, head_dim, theta, str(device), None if llama3 is None else tuple(sorted(llama3.items())))
    t = _ROPE_CACHE.get(key)
    if t is None:
        t = R.rope_cos_sin(seq, head_dim, theta, device=device, llama3=llama3)
        _ROPE_CACHE[key] = t
    return t


def attention_block(h, x, w_qkv, attn_gate, w_o, shape: AttnShape, segment_ids=None):
    """``x + W_o( gate * XSA( attn( rope(qknorm(W_q h)), rope(qknorm(W_k h)), W_v h ) ) )``
    (megagpt-speedrun/model.py:255-285). ``h`` is the normalised block input, ``x`` the residual."""
    if h.is_cuda:
        return _cuda().attention_block(h, x, w_qkv, attn_gate, w_o, shape, segment_ids)
    b, s, nh, hkv, hd = shape.batch, shape.seq, shape.heads, shape.kv_heads, shape.head_dim
    qkv = h @ w_qkv.t()
    q = qkv[:, : shape.q_cols].reshape(b, s, nh, hd)
    k = qkv[:, shape.q_cols: shape.q_cols + shape.kv_cols].reshape(b, s, hkv, hd)
    v = qkv[:, shape.q_cols + shape.kv_cols:].reshape(b, s, hkv, hd)
    if shape.qk_norm:
        q = R.rms_norm_noparam(q)
        k = R.rms_norm_noparam(k)
    cos, sin = rope_tables(s, hd, shape.rope_theta, h.device, shape.llama3)
    q = R.apply_rope(q, cos, sin)
    k = R.apply_rope(k, cos, sin)
    q = q * shape.qk_mult
    seg = None if segment_ids is None else segment_ids.view(b, s)
    o = R.attention(q, k, v, window=shape.window, segment_ids=seg)
    if shape.xsa or shape.head_gate:
        gate_w = attn_gate if attn_gate is not None else torch.zeros(nh, h.shape[1], device=h.device)
        o = R.xsa_head_gate(o, v, h.view(b, s, -1), gate_w, xsa=shape.xsa, head_gate=shape.head_gate)
    o = o.reshape(b * s, nh * hd)
    return x + o @ w_o.t()


# -------------------------------------------------------------------------------------- MLPs


def dense_mlp(h, w_in, w_down, *, glu: bool, act: str, residual=None):
    """Dense MLP: SwiGLU (blocked gate/up rows in ``w_in``) or plain ``act(h W_in^T) W_down^T``."""
    if h.is_cuda:
        return _cuda().dense_mlp(h, w_in, w_down, glu, act, residual)
    z = h @ w_in.t()
    if glu:
        g, u = split_gate_up(z, w_down.shape[1])
        a = R.activation(g, act) * u
    else:
        a = R.activation(z, act)
    y = a @ w_down.t()
    return y if residual is None else residual + y


# ------------------------------------------------------------------------------------ router


class RouterOut:
    """Routing decision and the differentiable router losses of one MoE layer."""

    def __init__(self, selected, combine, keep, z_loss, lbl, sparsity, counts, entropy, beta, expected, realized):
        self.selected, self.combine, self.keep = selected, combine, keep
        self.z_loss, self.lbl, self.sparsity = z_loss, lbl, sparsity
        self.counts, self.entropy, self.beta = counts, entropy, beta
        self.expected_active, self.realized_active = expected, realized


def route(h, w_router, router_bias, k: int, *, adaptive=False, threshold=None, k_min=0, temp=1.0,
          qb_count: int = 1, need_beta: bool = True, logit_bias=None):
    """Router of megagpt-speedrun/model.py:559-634: fp32 logits, top-(K+1) on biased logits,
    sigmoid combine weights on unbiased logits, per-layer z-loss / LBL / sparsity penalty and the
    local QB beta (the cross-rank mean is taken by the caller). ``logit_bias`` ``[E]`` is an optional
    learned additive logit bias (depth-conditioned routing), differentiated like the logits."""
    if h.is_cuda:
        return _cuda().route(h, w_router, router_bias, k, adaptive, threshold, k_min, temp, qb_count, need_beta,
                             logit_bias)
    out = R.route(h, w_router, router_bias, k, adaptive=adaptive, threshold=threshold, k_min=k_min, temp=temp,
                  logit_bias=logit_bias)
    e = w_router.shape[0]
    st = R.routing_stats(out["selected"], out["probs"], out["logits"], e, k)
    beta = R.qb_beta(out["logits"].detach(), out["alpha"].detach(), qb_count) if need_beta else None
    sparsity = out["expected_active"].mean() / e
    return RouterOut(out["selected"], out["combine"], out["hard_keep"], st["router_z_loss"],
                     st["load_balancing_loss"], sparsity, st["routing_counts"], st["routing_entropy"], beta,
                     out["expected_active"].mean() / e, out["realized_active"].mean() / e)


def moe_experts(h, r: RouterOut, w_gate_up, w_down, *, capacity: int | None, act: str = "silu", residual=None):
    """Routed expert SwiGLU MLP over the capacity layout (``capacity=None``: dropless)."""
    if h.is_cuda:
        return _cuda().moe_experts(h, r, w_gate_up, w_down, capacity, act, residual)
    from .layout import blocked_rows_to_gate_up

    g, u = blocked_rows_to_gate_up(w_gate_up)
    w_std = torch.cat([g, u], dim=1)
    keep = r.keep if not bool(r.keep.all()) else None
    y = R.moe_experts(h, r.selected, r.combine, w_std, w_down, capacity=capacity, keep=keep, act=act)
    return y if residual is None else residual + y


def capacity_for(tokens: int, k: int, experts: int, factor: float, align: int = 128) -> int:
    """Per-expert buffer rows: ceil(factor * tokens * k / experts) rounded up to ``align``."""
    c = int(math.ceil(factor * tokens * k / experts))
    return max(align, (c + align - 1) // align * align)


# ------------------------------------------------------------------------------------- loss


def cross_entropy(h, w_out, labels, weights, *, z_weight: float = 0.0):
    """Fused linear + softmax cross-entropy with z-loss; weighted mean over tokens."""
    if h.is_cuda:
        return _cuda().cross_entropy(h, w_out, labels, weights, z_weight)
    return R.fused_linear_cross_entropy(h, w_out, labels, weights, z_weight=z_weight)


def ngram_embed(ids: torch.Tensor, table: torch.Tensor, orders, n_hash: int) -> torch.Tensor:
    """Hashed n-gram input embedding ``[B*S, rank]`` (mean over orders x hashes)."""
    if ids.is_cuda:
        return _cuda().ngram_embed(ids, table, orders, n_hash)
    return R.ngram_embed(ids, table, orders, n_hash)
