"""Autograd Functions over the sm_100a kernels (the CUDA path of ``ops.api``).

Weight gradients are accumulated in fp32 directly into ``param.main_grad`` by the GEMM epilogues
(a ``main_grad`` buffer is created on first use when the parameter store has not attached one),
and the Functions return ``None`` for those inputs. 2-D+ weights are bf16 compute copies; 1-D
parameters (norm scales, router bias, thresholds) are fp32.
"""

from __future__ import annotations

import math

import torch

from . import gemm as G
from ._ext import ext

BF16 = torch.bfloat16
F32 = torch.float32


def _mg(p: torch.Tensor) -> torch.Tensor:
    g = getattr(p, "main_grad", None)
    if g is None:
        g = torch.zeros(p.shape, dtype=F32, device=p.device)
        p.main_grad = g
    return g


def _round(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------------- embedding


class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table):
        ids = _c(ids.long())
        out = torch.empty(ids.numel(), table.shape[1], dtype=BF16, device=ids.device)
        ext().embed_fwd(ids, table, out)
        ctx.save_for_backward(ids)
        ctx.table = table
        return out

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        ext().embed_bwd(ids, _c(dout), _mg(ctx.table))
        ctx.table = None
        return None, None


def embed(ids, table):
    return _Embed.apply(ids, table)


# ------------------------------------------------------------------------------------- linear


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual):
        x = _c(x)
        if residual is not None:
            out = torch.empty(x.shape[0], w.shape[0], dtype=BF16, device=x.device)
            G.linear(x, w, out=out, epi="resid", r=_c(residual))
        else:
            out = G.linear(x, w)
        ctx.save_for_backward(x)
        ctx.w = w
        ctx.has_res = residual is not None
        return out

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        w = ctx.w
        dy = _c(dy)
        dx = G.linear_dx(dy, w)
        G.linear_dw(dy, x, out=_mg(w), accum=True)
        ctx.w = None
        return dx, None, (dy if ctx.has_res else None)


def linear(x, w, residual=None):
    return _Linear.apply(x, w, residual)


# -------------------------------------------------------------------------------- norms


class _RmsGatedNorm(torch.autograd.Function):
    """RMSNorm (+ GatedNorm). With ``passthrough`` it also returns an alias of ``x`` to be used as
    the block's residual: the residual's gradient then arrives here and is added inside the RMSNorm
    backward kernel instead of by a separate autograd accumulation."""

    @staticmethod
    def forward(ctx, x, w_rms, eps, w_down, w_up, passthrough=False):
        x = _c(x)
        t, d = x.shape
        y = torch.empty_like(x)
        rstd = torch.empty(t, dtype=F32, device=x.device)
        ext().rmsnorm_fwd(x, w_rms, y, rstd, eps)
        ctx.gated = w_down is not None
        ctx.w_rms = w_rms
        ctx.set_materialize_grads(False)  # a missing residual gradient is passed on as None
        if not ctx.gated:
            ctx.save_for_backward(x, rstd)
            return (y, x.view_as(x)) if passthrough else y
        r = w_down.shape[0]
        s = torch.empty(t, r, dtype=BF16, device=x.device)
        h = torch.empty(t, r, dtype=BF16, device=x.device)
        G.gemm(y, w_down, s, M=t, N=r, K=d, epi="silu", c2=h)
        out = torch.empty_like(x)
        G.gemm(s, w_up, out, M=t, N=d, K=r, epi="gate_mul", r=y)
        ctx.save_for_backward(x, rstd, y, h, s)
        ctx.w_down, ctx.w_up = w_down, w_up
        return (out, x.view_as(x)) if passthrough else out

    @staticmethod
    def backward(ctx, dout, dres=None):
        if dout is None:
            dout = torch.zeros_like(ctx.saved_tensors[0])
        dout = _c(dout)
        dres = None if dres is None else _c(dres)
        if not ctx.gated:
            x, rstd = ctx.saved_tensors
            dy = dout
        else:
            x, rstd, y, h, s = ctx.saved_tensors
            w_down, w_up = ctx.w_down, ctx.w_up
            t, d = x.shape
            r = w_down.shape[0]
            z = torch.empty_like(x)
            G.gemm(s, w_up, z, M=t, N=d, K=r)
            dy1 = torch.empty_like(x)
            dz = torch.empty_like(x)
            ext().gate_mul_bwd(dout, y, z, dy1, dz)
            del z
            G.linear_dw(dz, s, out=_mg(w_up), accum=True)
            ds = G.linear_dx(dz, w_up)
            dh = torch.empty_like(ds)
            ext().act_bwd(ds, h, dh, 0)
            G.linear_dw(dh, y, out=_mg(w_down), accum=True)
            dy = torch.empty_like(x)
            G.gemm(dh, w_down, dy, b_mn=True, M=t, N=d, K=r, epi="resid", r=dy1)
            ctx.w_down = ctx.w_up = None
        dx = torch.empty_like(x)
        ext().rmsnorm_bwd(dy, x, ctx.w_rms, rstd, dres, dx, _mg(ctx.w_rms))
        ctx.w_rms = None
        return dx, None, None, None, None, None


def rms_gated_norm(x, w_rms, eps, w_down=None, w_up=None, passthrough=False):
    return _RmsGatedNorm.apply(x, w_rms, eps, w_down, w_up, passthrough)


# ---------------------------------------------------------------------------------- attention


def _qkvg_weight(w_qkv, attn_gate):
    """The [q | k | v | gate] weight rows as one matrix (and its main_grad view).

    The parameter store lays ``attn_gate`` out directly after ``w_qkv``; the fused view is then
    free. Standalone tensors fall back to a concatenated copy whose gradient is split back."""
    if attn_gate is None:
        return w_qkv, None
    fused = getattr(w_qkv, "_qkvg_view", None)
    if fused is not None:
        return fused, None
    return torch.cat([w_qkv, attn_gate], dim=0), (w_qkv.shape[0],)


class _AttentionBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, x, w_qkv, attn_gate, w_o, shape, seg):
        from .api import rope_tables

        h = _c(h)
        t, d = h.shape
        nh, hkv, hd, s = shape.heads, shape.kv_heads, shape.head_dim, shape.seq
        nq, nk = nh * hd, hkv * hd
        use_gate = shape.head_gate and attn_gate is not None
        W, split = _qkvg_weight(w_qkv, attn_gate if use_gate else None)
        n = W.shape[0]
        ld = _round(n, 64)
        qkvg = torch.empty(t, ld, dtype=BF16, device=h.device)
        G.gemm(h, W, qkvg, M=t, N=n, K=d)
        cos, sin = rope_tables(s, hd, shape.rope_theta, h.device, shape.llama3)
        qn = torch.empty(t, nh, hd, dtype=BF16, device=h.device)
        kn = torch.empty(t, hkv, hd, dtype=BF16, device=h.device)
        rstd = torch.empty(t, nh + hkv, dtype=F32, device=h.device)
        ext().qk_norm_rope_fwd(qkvg, qn, kn, rstd, cos, sin, s, nh, hkv, hd, shape.qk_norm, shape.qk_mult)
        v = qkvg[:, nq + nk: nq + 2 * nk].view(t, hkv, hd)
        o = torch.empty(t, nh, hd, dtype=BF16, device=h.device)
        lse = torch.empty(t, nh, dtype=F32, device=h.device)
        seg = None if seg is None else _c(seg.int())
        scale = 1.0 / math.sqrt(hd)
        if hd in (64, 96, 128):
            from ._ext import err_flag

            # tcgen05 forward (TMEM accumulators, TMA-fed); segments must be contiguous runs
            ext().flash_fwd_sm100(qn, kn, v, o, lse, seg, shape.batch, s, shape.window, scale, err_flag(h.device),
                                  None)
        else:
            ext().flash_fwd(qn, kn, v, o, lse, seg, shape.batch, s, shape.window, scale)
        if shape.xsa or use_gate:
            o2 = torch.empty(t, nq, dtype=BF16, device=h.device)
            ext().xsa_gate_fwd(o, qkvg, nq + nk, nq + 2 * nk, o2, nh, hkv, hd, shape.xsa, use_gate)
        else:
            o2 = o.view(t, nq)
        out = torch.empty(t, d, dtype=BF16, device=h.device)
        G.linear(o2, w_o, out=out, epi="resid", r=_c(x))
        ctx.save_for_backward(h, qkvg, qn, kn, rstd, o, lse, o2, cos, sin)
        ctx.seg = seg
        ctx.W, ctx.split, ctx.w_qkv, ctx.attn_gate, ctx.w_o = W, split, w_qkv, attn_gate, w_o
        ctx.shape, ctx.use_gate, ctx.n, ctx.scale = shape, use_gate, n, scale
        return out

    @staticmethod
    def backward(ctx, dout):
        h, qkvg, qn, kn, rstd, o, lse, o2, cos, sin = ctx.saved_tensors
        shape = ctx.shape
        dout = _c(dout)
        t, d = h.shape
        nh, hkv, hd, s = shape.heads, shape.kv_heads, shape.head_dim, shape.seq
        nq, nk = nh * hd, hkv * hd
        do2 = G.linear_dx(dout, ctx.w_o)
        G.linear_dw(dout, o2, out=_mg(ctx.w_o), accum=True)
        ld = qkvg.shape[1]
        dqkvg = torch.empty(t, ld, dtype=BF16, device=h.device)
        if ld > ctx.n:
            dqkvg[:, ctx.n:].zero_()
        dv = dqkvg[:, nq + nk: nq + 2 * nk].view(t, hkv, hd)
        if shape.xsa or ctx.use_gate:
            do = torch.empty(t, nh, hd, dtype=BF16, device=h.device)
            ext().xsa_gate_bwd(do2, o, qkvg, nq + nk, nq + 2 * nk, do, dqkvg, nh, hkv, hd, shape.xsa, ctx.use_gate)
            dv_acc = True
        else:
            do = do2.view(t, nh, hd)
            dv_acc = False
        v = qkvg[:, nq + nk: nq + 2 * nk].view(t, hkv, hd)
        dq = torch.empty(t, nh, hd, dtype=BF16, device=h.device)
        dk = torch.empty(t, hkv, hd, dtype=BF16, device=h.device)
        dq_acc = torch.empty(t, nh, hd, dtype=F32, device=h.device)
        dsum = torch.empty(t, nh, dtype=F32, device=h.device)
        if hd in (64, 96, 128) and s < 32767:
            from ._ext import err_flag

            ext().flash_bwd_sm100(qn, kn, v, o, lse, ctx.seg, shape.batch, s, shape.window, ctx.scale, _c(do), dsum,
                                  dq_acc, dq, dk, dv, dv_acc, err_flag(h.device))
        else:
            ext().flash_bwd(qn, kn, v, o, lse, ctx.seg, shape.batch, s, shape.window, ctx.scale, _c(do), dsum, dq_acc,
                            dq, dk, dv, dv_acc)
        ext().qk_norm_rope_bwd(dq, dk, qkvg, rstd, cos, sin, dqkvg, s, nh, hkv, hd, shape.qk_norm, shape.qk_mult)
        W = ctx.W
        dh = torch.empty(t, d, dtype=BF16, device=h.device)
        G.gemm(dqkvg, W, dh, b_mn=True, M=t, N=d, K=ld)
        n_rows = ctx.n
        if ctx.split is None:
            wg = getattr(ctx.w_qkv, "_qkvg_grad", None)
            if wg is None:
                wg = _mg(ctx.w_qkv)
            G.weight_grad(lambda: G.gemm(dqkvg, h, wg, a_mn=True, b_mn=True, M=n_rows, N=d, K=t, accum=True))
        else:
            r0 = ctx.split[0]
            gq, gg = _mg(ctx.w_qkv), _mg(ctx.attn_gate)

            def _dw_split():
                tmp = torch.zeros(n_rows, d, dtype=F32, device=h.device)
                G.gemm(dqkvg, h, tmp, a_mn=True, b_mn=True, M=n_rows, N=d, K=t, accum=True)
                gq.add_(tmp[:r0])
                gg.add_(tmp[r0:])

            G.weight_grad(_dw_split)
        ctx.W = ctx.w_qkv = ctx.attn_gate = ctx.w_o = None
        return dh, dout, None, None, None, None, None


def attention_block(h, x, w_qkv, attn_gate, w_o, shape, seg):
    return _AttentionBlock.apply(h, x, w_qkv, attn_gate, w_o, shape, seg)


# ----------------------------------------------------------------------------------- MLPs

_ACT = {"silu": 0, "relu": 1, "gelu": 2}


class _DenseMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w_in, w_down, glu, act, residual):
        h = _c(h)
        t, d = h.shape
        inter = w_down.shape[1]
        if glu:
            H = torch.empty(t, 2 * inter, dtype=BF16, device=h.device)
            A = torch.empty(t, inter, dtype=BF16, device=h.device)
            G.gemm(h, w_in, H, M=t, N=2 * inter, K=d, epi="swiglu", c2=A)
        else:
            H = torch.empty(t, inter, dtype=BF16, device=h.device)
            A = torch.empty(t, inter, dtype=BF16, device=h.device)
            G.gemm(h, w_in, A, M=t, N=inter, K=d, epi="act", c2=H, act=act)
        out = torch.empty(t, d, dtype=BF16, device=h.device)
        if residual is not None:
            G.gemm(A, w_down, out, M=t, N=d, K=inter, epi="resid", r=_c(residual))
        else:
            G.gemm(A, w_down, out, M=t, N=d, K=inter)
        ctx.save_for_backward(h, H, A)
        ctx.w_in, ctx.w_down, ctx.glu, ctx.act, ctx.has_res = w_in, w_down, glu, act, residual is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        h, H, A = ctx.saved_tensors
        dout = _c(dout)
        if ctx.glu and ctx.act == "silu":
            # the activation-gradient GEMM writes the gate/up gradients in its epilogue
            dH = G.linear_dx(dout, ctx.w_down, swiglu_h=H)
            G.linear_dw(dout, A, out=_mg(ctx.w_down), accum=True)
        else:
            dA = G.linear_dx(dout, ctx.w_down)
            G.linear_dw(dout, A, out=_mg(ctx.w_down), accum=True)
            dH = torch.empty_like(H)
            if ctx.glu:
                ext().swiglu_bwd(dA, H, dH, _ACT[ctx.act], None, 0)
            else:
                ext().act_bwd(dA, H, dH, _ACT[ctx.act])
        dh = G.linear_dx(dH, ctx.w_in)
        G.linear_dw(dH, h, out=_mg(ctx.w_in), accum=True)
        ctx.w_in = ctx.w_down = None
        return dh, None, None, None, None, (dout if ctx.has_res else None)


def dense_mlp(h, w_in, w_down, glu, act, residual):
    return _DenseMLP.apply(h, w_in, w_down, glu, act, residual)


# --------------------------------------------------------------------------------- router


class _Router(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w_router, theta, bias, k, adaptive, k_min, temp, qb_count, need_beta, logit_bias):
        h = _c(h)
        t, d = h.shape
        e = w_router.shape[0]
        dev = h.device
        ldl = _round(e, 32)
        logits = torch.empty(t, ldl, dtype=F32, device=dev)
        G.gemm(h, w_router, logits, M=t, N=e, K=d, bn=64)
        if logit_bias is not None:
            logits[:, :e] += logit_bias.detach().float()
        ctx.has_lb = logit_bias is not None
        sel = torch.empty(t, k, dtype=torch.int32, device=dev)
        comb = torch.empty(t, k, dtype=F32, device=dev)
        topb = torch.empty(t, k, dtype=F32, device=dev)
        alpha = torch.empty(t, dtype=F32, device=dev)
        lse = torch.empty(t, dtype=F32, device=dev)
        keep = torch.empty(t, k, dtype=torch.uint8, device=dev)
        acc = torch.zeros(2 * e + 3, dtype=F32, device=dev)
        counts, psum, scal = acc[:e], acc[e:2 * e], acc[2 * e:]
        th = (theta.detach().float().reshape(1) if theta is not None
              else torch.zeros(1, dtype=F32, device=dev))
        ext().router_fwd(logits, bias.detach().float(), e, k, adaptive, th, k_min, temp, sel, comb, topb, alpha, lse,
                         keep, counts, psum, scal)
        z_loss = scal[0] / t
        lbl = e * ((counts / t) * (psum / t)).sum()
        sparsity = scal[1] / (t * e)
        realized = scal[2] / (t * e)
        frac = counts / counts.sum().clamp_min(1.0)
        entropy = -(frac * torch.log(frac + 1e-6)).sum()
        beta = None
        if need_beta:
            beta = torch.empty(e, dtype=F32, device=dev)
            ext().qb_beta(logits, alpha, e, qb_count, beta)
        ctx.save_for_backward(h, logits, lse, sel, topb, keep, counts, th)
        ctx.w_router, ctx.theta = w_router, theta
        ctx.k, ctx.adaptive, ctx.k_min, ctx.temp, ctx.e = k, adaptive, k_min, temp, e
        # unused outputs (statistics, an auxiliary loss with weight 0) get no zero-filled gradient
        # tensors: the backward treats a missing gradient as zero
        ctx.set_materialize_grads(False)
        ctx.mark_non_differentiable(sel, keep, counts, entropy, realized)
        if beta is not None:
            ctx.mark_non_differentiable(beta)
        return comb, z_loss, lbl, sparsity, sel, keep, counts, entropy, realized, beta

    @staticmethod
    def backward(ctx, dcomb, dz, dlbl, dsp, *_):
        h, logits, lse, sel, topb, keep, counts, th = ctx.saved_tensors
        t, d = h.shape
        e = ctx.e
        dev = h.device
        zero = torch.zeros((), dtype=F32, device=dev)
        dscal = torch.stack([(dz if dz is not None else zero).float().reshape(()),
                             (dlbl if dlbl is not None else zero).float().reshape(()),
                             (dsp if dsp is not None else zero).float().reshape(())])
        if dcomb is None:
            dcomb = torch.zeros(t, ctx.k, dtype=F32, device=dev)
        ldd = _round(e, 64)
        dlog = torch.empty(t, ldd, dtype=BF16, device=dev)
        dtheta = torch.zeros(1, dtype=F32, device=dev)
        ext().router_bwd(logits, lse, sel, topb, keep, _c(dcomb.float()), counts, dscal, e, ctx.k, ctx.adaptive, th,
                         ctx.k_min, ctx.temp, dlog, dtheta)
        dh = torch.empty(t, d, dtype=BF16, device=dev)
        G.gemm(dlog, ctx.w_router, dh, b_mn=True, M=t, N=d, K=ldd)
        gr = _mg(ctx.w_router)
        G.weight_grad(lambda: G.gemm(dlog, h, gr, a_mn=True, b_mn=True, M=e, N=d, K=t, accum=True))
        if ctx.adaptive and ctx.theta is not None:
            _mg(ctx.theta).add_(dtheta.reshape(_mg(ctx.theta).shape))
        ctx.w_router = ctx.theta = None
        dlb = dlog[:, :e].float().sum(0) if ctx.has_lb else None
        return dh, None, None, None, None, None, None, None, None, None, dlb


def route(h, w_router, router_bias, k, adaptive, threshold, k_min, temp, qb_count, need_beta, logit_bias=None):
    from .api import RouterOut

    comb, z_loss, lbl, sparsity, sel, keep, counts, entropy, realized, beta = _Router.apply(
        h, w_router, threshold, router_bias, k, adaptive, k_min, temp, qb_count, need_beta, logit_bias)
    e = w_router.shape[0]
    return RouterOut(sel, comb, keep.bool(), z_loss, lbl, sparsity, counts, entropy, beta, sparsity.detach(),
                     realized)


# ------------------------------------------------------------------------------------- MoE


def dispatch_plan(sel, keep, comb, e: int, cap: int):
    """Capacity-layout plan: per-assignment slot (-1 = dropped), per-slot token and combine
    weight, per-expert kept counts."""
    t, k = sel.shape
    dev = sel.device
    ws = torch.empty(ext().plan_workspace(t * k, e), dtype=torch.int32, device=dev)
    slot = torch.empty(t, k, dtype=torch.int32, device=dev)
    perm = torch.empty(e * cap, dtype=torch.int32, device=dev)
    wperm = torch.empty(e * cap, dtype=F32, device=dev)
    counts = torch.empty(e, dtype=torch.int32, device=dev)
    ext().dispatch_plan(_c(sel), keep, _c(comb.detach().float()), e, cap, ws, slot, perm, wperm, counts)
    return slot, perm, wperm, counts


class _MoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, comb, w_gu, w_d, residual, sel, keep, cap, act):
        h = _c(h)
        t, d = h.shape
        e, two_i, _ = w_gu.shape
        inter = two_i // 2
        dev = h.device
        slot, perm, wperm, counts = dispatch_plan(sel, keep, comb, e, cap)
        xp = torch.empty(e * cap, d, dtype=BF16, device=dev)
        ext().permute(h, perm, counts, cap, xp)
        Hh = torch.empty(e * cap, two_i, dtype=BF16, device=dev)
        A = torch.empty(e * cap, inter, dtype=BF16, device=dev)
        G.grouped_linear(xp, w_gu.view(e * two_i, d), counts, out=Hh, epi="swiglu", c2=A)
        Y = G.grouped_linear(A, w_d.view(e * d, inter), counts)
        out = torch.empty(t, d, dtype=BF16, device=dev)
        ext().combine(Y, sel, slot, _c(comb.detach().float()), None if residual is None else _c(residual), out, cap)
        ctx.save_for_backward(xp, Hh, A, Y, sel, slot, perm, wperm, counts)
        ctx.w_gu, ctx.w_d, ctx.cap, ctx.has_res, ctx.act, ctx.t = w_gu, w_d, cap, residual is not None, act, t
        return out

    @staticmethod
    def backward(ctx, dout):
        xp, Hh, A, Y, sel, slot, perm, wperm, counts = ctx.saved_tensors
        dout = _c(dout)
        w_gu, w_d, cap = ctx.w_gu, ctx.w_d, ctx.cap
        e, two_i, d = w_gu.shape
        inter = two_i // 2
        dev = dout.device
        dY = torch.empty_like(Y)
        dcomb = torch.empty(sel.shape, dtype=F32, device=dev)
        ext().combine_bwd(dout, Y, sel, slot, perm, wperm, counts, cap, dY, dcomb)
        if ctx.act == "silu":
            dH = G.grouped_linear_dx(dY, w_d.view(e * d, inter), counts, swiglu_h=Hh)
            G.grouped_linear_dw(dY, A, counts, out=_mg(w_d).view(e * d, inter))
        else:
            dA = G.grouped_linear_dx(dY, w_d.view(e * d, inter), counts)
            G.grouped_linear_dw(dY, A, counts, out=_mg(w_d).view(e * d, inter))
            dH = torch.empty_like(Hh)
            ext().swiglu_bwd(dA, Hh, dH, _ACT[ctx.act], counts, cap)
        dxp = G.grouped_linear_dx(dH, w_gu.view(e * two_i, d), counts)
        G.grouped_linear_dw(dH, xp, counts, out=_mg(w_gu).view(e * two_i, d))
        dh = torch.empty(ctx.t, d, dtype=BF16, device=dev)
        ext().unpermute_add(dxp, sel, slot, None, dh, cap)
        ctx.w_gu = ctx.w_d = None
        return dh, dcomb, None, None, (dout if ctx.has_res else None), None, None, None, None


def moe_experts(h, r, w_gate_up, w_down, capacity, act, residual):
    t = h.shape[0]
    k = r.selected.shape[1]
    cap = capacity if capacity is not None else _round(t, 128)
    keep = None if r.keep is None else r.keep.to(torch.uint8)
    return _MoE.apply(h, r.combine, w_gate_up, w_down, residual, r.selected, keep, cap, act)


# ----------------------------------------------------------------------------- cross-entropy


class _CrossEntropy(torch.autograd.Function):
    """Fused linear + softmax cross-entropy. The gradient is computed in the forward pass, chunk
    by chunk over tokens (logits never exist for more than ``chunk`` tokens): the LM-head weight
    gradient is accumulated into ``main_grad`` with the factor ``grad_scale`` and the hidden-state
    gradient is kept for backward. Backward therefore requires the incoming gradient to equal
    ``grad_scale`` (the trainer's per-microbatch loss scale), and rescales dH by their ratio."""

    @staticmethod
    def forward(ctx, h, w, labels, weights, z_weight, grad_scale, chunk):
        h = _c(h)
        t, de = h.shape
        v = w.shape[0]
        dev = h.device
        nt = (v + 255) // 256
        vpad = nt * 256
        labels = _c(labels.long())
        weights = _c(weights.float())
        wsum = weights.sum().reshape(1)
        loss = torch.zeros(1, dtype=F32, device=dev)
        dH = torch.empty(t, de, dtype=BF16, device=dev)
        tc = min(chunk, t)
        logits = torch.empty(tc, vpad, dtype=BF16, device=dev)
        stats = torch.empty(tc, 4 * nt, dtype=F32, device=dev)  # (max, sumexp) per tile half
        wg = _mg(w)
        for c0 in range(0, t, tc):
            n = min(tc, t - c0)
            hc = h[c0:c0 + n]
            lg = logits[:n]
            st = stats[:n]
            G.gemm(hc, w, lg, M=n, N=v, K=de, epi="ce", c2=st)
            ext().ce_grad(lg, st, labels[c0:c0 + n], weights[c0:c0 + n], wsum, loss, None, v, z_weight, grad_scale)
            G.gemm(lg, w, dH[c0:c0 + n], b_mn=True, M=n, N=de, K=vpad)
            if n % 64 == 0:
                G.gemm(lg, hc, wg, a_mn=True, b_mn=True, M=v, N=de, K=n, accum=True)
            else:
                raise ValueError("token chunk must be a multiple of 64")
        ctx.save_for_backward(dH)
        ctx.grad_scale = grad_scale
        return (loss / wsum.clamp_min(1.0)).reshape(())

    @staticmethod
    def backward(ctx, g):
        (dH,) = ctx.saved_tensors
        ratio = g.float() / ctx.grad_scale
        return (dH * ratio).to(BF16), None, None, None, None, None, None


_CE_GRAD_SCALE = [1.0]


def set_loss_grad_scale(scale: float) -> None:
    """Declare the gradient the CE loss will receive in backward (1 / #microbatches)."""
    _CE_GRAD_SCALE[0] = float(scale)


@torch.no_grad()
def _ce_loss_only(h, w, labels, weights, z_weight, chunk):
    """Evaluation path: the same fused GEMM + softmax epilogue, no gradient GEMMs (and no write
    into the weight's ``main_grad``)."""
    h = _c(h)
    t, _ = h.shape
    v = w.shape[0]
    nt = (v + 255) // 256
    labels = _c(labels.long())
    weights = _c(weights.float())
    wsum = weights.sum().reshape(1)
    loss = torch.zeros(1, dtype=F32, device=h.device)
    tc = min(chunk, t)
    logits = torch.empty(tc, nt * 256, dtype=BF16, device=h.device)
    stats = torch.empty(tc, 4 * nt, dtype=F32, device=h.device)
    for c0 in range(0, t, tc):
        n = min(tc, t - c0)
        G.gemm(h[c0:c0 + n], w, logits[:n], M=n, N=v, K=h.shape[1], epi="ce", c2=stats[:n])
        ext().ce_grad(logits[:n], stats[:n], labels[c0:c0 + n], weights[c0:c0 + n], wsum, loss, None, v,
                      float(z_weight), 1.0)
    return (loss / wsum.clamp_min(1.0)).reshape(())


def cross_entropy(h, w_out, labels, weights, z_weight, chunk: int = 8192):
    if not torch.is_grad_enabled() or not (h.requires_grad or w_out.requires_grad):
        return _ce_loss_only(h, w_out, labels, weights, z_weight, chunk)
    return _CrossEntropy.apply(h, w_out, labels, weights, float(z_weight), _CE_GRAD_SCALE[0], chunk)


# ------------------------------------------------------------------------ hashed n-gram embedding
class _NgramEmbed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table, orders, n_hash):
        ids = _c(ids.long())
        b, s = ids.shape
        o, buckets, rank = table.shape
        ords = torch.tensor(list(orders), dtype=torch.int32, device=ids.device)
        out = torch.empty(b * s, rank, dtype=BF16, device=ids.device)
        ext().ngram_fwd(ids, ords, n_hash, buckets, _c(table), out)
        ctx.save_for_backward(ids, ords)
        ctx.table, ctx.n_hash, ctx.buckets = table, n_hash, buckets
        return out

    @staticmethod
    def backward(ctx, dout):
        ids, ords = ctx.saved_tensors
        ext().ngram_bwd(ids, ords, ctx.n_hash, ctx.buckets, _c(dout), _mg(ctx.table))
        ctx.table = None
        return None, None, None, None


def ngram_embed(ids, table, orders, n_hash):
    return _NgramEmbed.apply(ids, table, tuple(orders), int(n_hash))
