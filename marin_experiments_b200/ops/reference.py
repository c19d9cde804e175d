"""Plain-PyTorch fp32 oracle for every hot op.

Each function here is the mathematical definition that the sm_100a kernels are tested against
(and the path the model takes on CPU). All functions are differentiable through torch
autograd, so the hand-written backward passes in ``ops.functional`` are checked against
autograd of these definitions.

Weight layout: linear weights are stored ``[out_features, in_features]`` (``y = x @ W.T``);
expert weights are ``w_gate_up [E, 2I, D]`` and ``w_down [E, D, I]``.

Semantics follow the reference model (megagpt-speedrun/model.py):
* ``rms_norm`` -- parametric RMSNorm in fp32 (model.py:288-303); ``rms_norm_noparam`` is the
  QK norm (model.py:228-231, eps 1e-6).
* ``gated_norm`` -- x * sigmoid(silu(x W_down) W_up) (model.py:306-328).
* ``apply_rope`` -- rotate-half rotary embedding (levanter ``apply_rotary_embedding``).
* ``attention`` -- causal softmax attention with optional sliding window, packed segment ids
  and GQA (levanter ``attention``; window semantics of ``AttentionMask.with_sliding_window``).
* ``xsa_head_gate`` -- exclusive self-attention and 2*sigmoid head gate (model.py:276-283).
* ``route`` -- fp32 router: softmax, top-(K+1) on biased logits, sigmoid combine weights on
  unbiased logits, QB alpha, routing stats (model.py:559-645, 371-396).
* ``fused_linear_cross_entropy`` -- logits = h W^T, logsumexp, weighted NLL + z-loss
  (levanter ``fused_linear_softmax_cross_entropy_loss``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    dtype = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    y = xf * torch.rsqrt(var + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(dtype)


def rms_norm_noparam(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return rms_norm(x, None, eps)


def gated_norm(x: torch.Tensor, w_down: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """``w_down`` is ``[R, D]`` and ``w_up`` is ``[D, R]`` (out, in)."""
    hidden = F.silu(x @ w_down.t())
    gate = torch.sigmoid(hidden @ w_up.t())
    return x * gate.to(x.dtype)


def rope_cos_sin(seq_len: int, head_dim: int, theta: float, device=None, llama3: dict | None = None):
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64, device=device) / half))
    if llama3 is not None:
        inv_freq = llama3_scale_inv_freq(inv_freq, **llama3)
    pos = torch.arange(seq_len, dtype=torch.float64, device=device)
    ang = torch.outer(pos, inv_freq)
    return ang.cos().float(), ang.sin().float()


def llama3_scale_inv_freq(inv_freq, scaling_factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                          original_max_position=8192):
    """Llama-3 RoPE frequency scaling (the rule the Qwen3/Delphi patch applies,
    tunix-delphi-rl/models/delphi_patch.py:47-159)."""
    low_wl = original_max_position / low_freq_factor
    high_wl = original_max_position / high_freq_factor
    wavelen = 2 * math.pi / inv_freq
    scaled = torch.where(wavelen > low_wl, inv_freq / scaling_factor, inv_freq)
    smooth = (original_max_position / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
    mid = (1 - smooth) * scaled / scaling_factor + smooth * scaled
    is_mid = (wavelen >= high_wl) & (wavelen <= low_wl)
    return torch.where(is_mid, mid, scaled)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: ``[B, S, H, hd]``; cos/sin: ``[S, hd/2]`` (rotate-half convention)."""
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return out.to(x.dtype)


def attention_mask(seq_len: int, window: int = 0, segment_ids: torch.Tensor | None = None, device=None):
    """Boolean ``[B or 1, S, S]`` visibility: j <= i, i - j < window (if window > 0), same segment."""
    i = torch.arange(seq_len, device=device)[:, None]
    j = torch.arange(seq_len, device=device)[None, :]
    m = j <= i
    if window > 0:
        m = m & ((i - j) < window)
    m = m[None]
    if segment_ids is not None:
        m = m & (segment_ids[:, :, None] == segment_ids[:, None, :])
    return m


def attention(q, k, v, *, window: int = 0, segment_ids=None, scale: float | None = None):
    """q: ``[B, S, H, hd]``, k/v: ``[B, S, Hkv, hd]`` -> ``[B, S, H, hd]`` (fp32 math)."""
    b, s, h, hd = q.shape
    hkv = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(hd)
    rep = h // hkv
    kf = k.float().repeat_interleave(rep, dim=2)
    vf = v.float().repeat_interleave(rep, dim=2)
    scores = torch.einsum("bqhd,bkhd->bhqk", q.float(), kf) * scale
    mask = attention_mask(s, window, segment_ids, device=q.device)[:, None]
    scores = scores.masked_fill(~mask, float("-inf"))
    p = torch.softmax(scores, dim=-1)
    out = torch.einsum("bhqk,bkhd->bqhd", p, vf)
    return out.to(q.dtype)


def xsa_head_gate(y, v, x, attn_gate, *, xsa: bool = True, head_gate: bool = True):
    """y: ``[B,S,H,hd]`` attention output, v: ``[B,S,Hkv,hd]``, x: ``[B,S,D]`` block input,
    attn_gate: ``[H, D]``."""
    h = y.shape[2]
    yf = y.float()
    if xsa:
        vf = v.float().repeat_interleave(h // v.shape[2], dim=2)
        dot = (yf * vf).sum(-1, keepdim=True)
        vn = (vf * vf).sum(-1, keepdim=True)
        yf = yf - (dot / (vn + 1e-6)) * vf
    if head_gate:
        gate = 2 * torch.sigmoid(x.float() @ attn_gate.float().t())
        yf = yf * gate[..., None]
    return yf.to(y.dtype)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return (F.silu(gate.float()) * up.float()).to(gate.dtype)


def activation(x: torch.Tensor, kind: str) -> torch.Tensor:
    if kind == "silu":
        return F.silu(x)
    if kind == "relu":
        return F.relu(x)
    if kind == "gelu":
        return F.gelu(x, approximate="tanh")
    raise ValueError(kind)


def route(x_flat, router_w, router_bias, k: int, *, adaptive: bool = False, threshold=None,
          k_min: int = 0, temp: float = 1.0, logit_bias=None):
    """Fp32 router (megagpt-speedrun/model.py:559-605).

    Returns a dict with ``logits`` [T,E], ``probs``, ``selected`` [T,K] (descending biased logit),
    ``topk_biased`` [T,K], ``alpha`` [T,1] (the (K+1)-th biased logit), ``combine`` [T,K] and, in
    adaptive mode, ``expected_active``/``realized_active`` per token."""
    logits = (x_flat @ router_w.t()).float()
    if logit_bias is not None:  # learned additive bias (part of the logits, with gradient)
        logits = logits + logit_bias.float()
    biased = logits + router_bias.detach().float()
    probs = torch.softmax(logits, dim=-1)
    e = logits.shape[-1]
    kk = min(k + 1, e)
    vals, idx = torch.topk(biased, kk, dim=-1)
    if kk > k:
        alpha = vals[:, k:k + 1]
    else:
        alpha = torch.full_like(vals[:, :1], float("-inf"))
    topk_biased, selected = vals[:, :k], idx[:, :k]
    combine = torch.sigmoid(torch.gather(logits, 1, selected))
    out = {"logits": logits, "probs": probs, "selected": selected, "topk_biased": topk_biased,
           "alpha": alpha}
    if adaptive:
        theta = threshold
        hard = topk_biased > theta
        soft = torch.sigmoid((topk_biased - theta) / temp)
        if k_min > 0:
            floor = torch.arange(k, device=x_flat.device) < k_min
            hard = hard | floor[None]
            soft = torch.where(floor[None], torch.ones_like(soft), soft)
        keep = hard.float() + (soft - soft.detach())
        combine = combine * keep
        out["expected_active"] = soft.sum(1)
        out["realized_active"] = hard.float().sum(1)
        out["hard_keep"] = hard
    else:
        full = torch.full((x_flat.shape[0],), float(k), device=x_flat.device)
        out["expected_active"] = full
        out["realized_active"] = full
        out["hard_keep"] = torch.ones_like(selected, dtype=torch.bool)
    out["combine"] = combine
    return out


def routing_stats(selected, probs, logits, num_experts: int, k: int, keep=None):
    """Expert counts, entropy, load-balancing loss E*sum(f_i p_i), router z-loss
    (megagpt-speedrun/model.py:371-396)."""
    oh = F.one_hot(selected, num_experts).float()
    if keep is not None:
        oh = oh * keep[..., None].float()
    counts = oh.sum((0, 1))
    total = counts.sum().clamp_min(1.0)
    frac = counts / total
    entropy = -(frac * torch.log(frac + 1e-6)).sum()
    token_frac = frac * k
    p = probs.float().mean(0)
    lbl = num_experts * (token_frac * p).sum()
    z = torch.logsumexp(logits.float(), dim=-1)
    zloss = (z ** 2).mean()
    return {"routing_counts": counts, "routing_entropy": entropy, "load_balancing_loss": lbl,
            "router_z_loss": zloss}


def qb_beta(logits, alpha, qb_count: int):
    """Per-expert qb_count-th largest (logit - alpha) over tokens (model.py:606-634, local part)."""
    s = (logits - alpha).t()
    vals, _ = torch.topk(s, qb_count, dim=-1)
    return vals[:, -1]


def capacity_slots(selected: torch.Tensor, num_experts: int, capacity: int, keep=None):
    """Position of each (token, k) assignment inside its expert's buffer, in flattened token-major
    order; assignments at slot >= capacity (or with keep False) are dropped (slot = -1)."""
    t, k = selected.shape
    flat = selected.reshape(-1)
    oh = F.one_hot(flat, num_experts).to(torch.int64)
    if keep is not None:
        oh = oh * keep.reshape(-1, 1).to(torch.int64)
    pos = torch.cumsum(oh, 0) - oh
    slot = torch.gather(pos, 1, flat[:, None]).squeeze(1)
    valid = slot < capacity
    if keep is not None:
        valid = valid & keep.reshape(-1)
    slot = torch.where(valid, slot, torch.full_like(slot, -1))
    counts = torch.minimum(oh.sum(0), torch.full((num_experts,), capacity, dtype=torch.int64,
                                                   device=selected.device))
    return slot.view(t, k), counts


def moe_experts(x_flat, selected, combine, w_gate_up, w_down, *, capacity: int | None = None,
                keep=None, act: str = "silu"):
    """Routed expert SwiGLU MLP.  ``capacity=None`` is dropless."""
    t, k = selected.shape
    e = w_gate_up.shape[0]
    inter = w_down.shape[2]
    out = torch.zeros(t, x_flat.shape[1], dtype=torch.float32, device=x_flat.device)
    if capacity is not None:
        slots, _ = capacity_slots(selected, e, capacity, keep)
        valid = slots >= 0
    else:
        valid = torch.ones_like(selected, dtype=torch.bool) if keep is None else keep
    xf = x_flat.float()
    for ei in range(e):
        tok, kk = torch.nonzero((selected == ei) & valid, as_tuple=True)
        if tok.numel() == 0:
            continue
        h = xf[tok] @ w_gate_up[ei].float().t()
        g, u = h[:, :inter], h[:, inter:]
        a = activation(g, act) * u
        y = a @ w_down[ei].float().t()
        out.index_add_(0, tok, y * combine[tok, kk].float()[:, None])
    return out.to(x_flat.dtype)


def fused_linear_cross_entropy(h, w, labels, weight=None, *, z_weight: float = 0.0, reduction="mean"):
    """h: ``[T, De]``, w: ``[V, De]``. Returns weighted mean NLL (+ z_weight * lse^2)."""
    logits = (h.float() @ w.float().t())
    lse = torch.logsumexp(logits, dim=-1)
    nll = lse - torch.gather(logits, 1, labels[:, None].long()).squeeze(1)
    if z_weight:
        nll = nll + z_weight * lse * lse
    if weight is None:
        weight = torch.ones_like(nll)
    if reduction == "none":
        return nll * weight
    if reduction == "sum":
        return (nll * weight).sum()
    return (nll * weight).sum() / weight.sum().clamp_min(1.0)


def adamh_matrix_update(p, u, lr: float):
    """Scale-invariant AdamH step for one matrix (megagpt-speedrun/adamh.py:52-58):
    new = p - lr * u * |p| / max(|u|, 1e-10); returns new / |new| * |p|."""
    pn = p.norm()
    un = u.norm()
    new = p - lr * u * pn / un.clamp_min(1e-10)
    return new / new.norm() * pn


# ------------------------------------------------------------------------ hashed n-gram embedding
_M64 = (1 << 64) - 1


def ngram_buckets(ids: torch.Tensor, n: int, h: int, buckets: int) -> torch.Tensor:
    """Bucket of the n-gram ending at every position of ``ids [B, S]`` under hash function ``h``
    (FNV-1a-style 64-bit mix salted by (n, h); positions before the sequence start count as -1)."""
    import numpy as np

    a = ids.detach().cpu().numpy().astype(np.int64)
    with np.errstate(over="ignore"):
        x = np.full(a.shape, 0xcbf29ce484222325 ^ (((n * 131 + h + 1) * 0x9E3779B97F4A7C15) & _M64), dtype=np.uint64)
        prime = np.uint64(0x100000001B3)
        for i in range(n):
            v = np.full(a.shape, -1, dtype=np.int64)
            v[:, i:] = a[:, : a.shape[1] - i] if i else a
            x ^= v.astype(np.uint64)
            x *= prime
            x ^= x >> np.uint64(29)
    return torch.from_numpy((x % np.uint64(buckets)).astype(np.int64)).to(ids.device)


def ngram_embed(ids: torch.Tensor, table: torch.Tensor, orders, n_hash: int) -> torch.Tensor:
    """``[B*S, rank]``: mean over (order, hash) of ``table[order][bucket]``."""
    n_o, buckets, rank = table.shape
    acc = None
    for oi, n in enumerate(orders):
        for h in range(n_hash):
            rows = table[oi].index_select(0, ngram_buckets(ids, n, h, buckets).reshape(-1))
            acc = rows if acc is None else acc + rows
    return acc / (len(orders) * n_hash)
