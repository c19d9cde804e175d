"""Expert parallelism: routed-expert MLP with experts sharded over an ``ep`` process group.

Rank r owns experts ``[r*E_loc, (r+1)*E_loc)``. Each source rank plans its local tokens'
assignments into a per-(source, expert) capacity of ``cap`` rows (first come, first served in
token order; cap = ceil(cf * T * K / E) rounded up to 128), scatters them into a send buffer
laid out ``[dest rank][local expert][cap][D]`` (= the single-GPU ``[E][cap]`` capacity layout), and
one equal-split all-to-all delivers ``[source rank][local expert][cap][D]`` to every destination.
The destination runs the grouped expert GEMMs over ``W * E_loc`` ragged groups (group
``s*E_loc + e`` uses expert ``e``'s weights; weight gradients of groups sharing an expert accumulate
with atomics) and a second all-to-all returns the outputs, which the source combines with its
routing weights. Backward mirrors it (two more all-to-alls). Shapes are static; only the
per-(source, expert) counts travel as data (a small all-to-all).

This replaces the reference's ring EP (all-gather of every token to every expert shard, then
psum-scatter; grug-moe-pp/pipeline.py:198-245), which moves W times more activation bytes.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import api as ops


def _a2a(out: torch.Tensor, inp: torch.Tensor, group) -> torch.Tensor:
    t0 = _mark() if out.is_cuda else None
    dist.all_to_all_single(out, inp, group=group)
    _span(t0)
    return out


class _MoEEP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, comb, w_gu, w_d, residual, sel, keep, cap, group, act):
        from ..ops import gemm as G
        from ..ops._ext import ext
        from ..ops.cuda_fns import _ACT, _c, dispatch_plan

        h = _c(h)
        t, d = h.shape
        e_loc, two_i, _ = w_gu.shape
        inter = two_i // 2
        world = dist.get_world_size(group)
        e = e_loc * world
        dev = h.device
        slot, perm, wperm, counts = dispatch_plan(sel, keep, comb, e, cap)
        xp_send = torch.empty(e * cap, d, dtype=torch.bfloat16, device=dev)
        ext().permute(h, perm, counts, cap, xp_send)
        counts_recv = _a2a(torch.empty_like(counts), counts, group)
        xp_recv = _a2a(torch.empty_like(xp_send), xp_send, group)
        Hh = torch.empty(e * cap, two_i, dtype=torch.bfloat16, device=dev)
        A = torch.empty(e * cap, inter, dtype=torch.bfloat16, device=dev)
        G.grouped_linear(xp_recv, w_gu.view(e_loc * two_i, d), counts_recv, out=Hh, epi="swiglu", c2=A, n_w=e_loc)
        y_recv = G.grouped_linear(A, w_d.view(e_loc * d, inter), counts_recv, n_w=e_loc)
        y_send = _a2a(torch.empty_like(y_recv), y_recv, group)
        out = torch.empty(t, d, dtype=torch.bfloat16, device=dev)
        ext().combine(y_send, sel, slot, _c(comb.detach().float()), None if residual is None else _c(residual), out,
                      cap)
        ctx.save_for_backward(xp_recv, Hh, A, y_send, sel, slot, perm, wperm, counts, counts_recv)
        ctx.w_gu, ctx.w_d, ctx.cap, ctx.group, ctx.act, ctx.t = w_gu, w_d, cap, group, _ACT[act], t
        ctx.has_res = residual is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        from ..ops import gemm as G
        from ..ops._ext import ext
        from ..ops.cuda_fns import _c, _mg

        xp_recv, Hh, A, y_send, sel, slot, perm, wperm, counts, counts_recv = ctx.saved_tensors
        dout = _c(dout)
        w_gu, w_d, cap, group = ctx.w_gu, ctx.w_d, ctx.cap, ctx.group
        e_loc, two_i, d = w_gu.shape
        inter = two_i // 2
        dev = dout.device
        dy_send = torch.empty_like(y_send)
        dcomb = torch.empty(sel.shape, dtype=torch.float32, device=dev)
        ext().combine_bwd(dout, y_send, sel, slot, perm, wperm, counts, cap, dy_send, dcomb)
        dy_recv = _a2a(torch.empty_like(dy_send), dy_send, group)
        if ctx.act == 0:  # SiLU gate: the activation-gradient GEMM writes dH in its epilogue
            dH = G.grouped_linear_dx(dy_recv, w_d.view(e_loc * d, inter), counts_recv, n_w=e_loc, swiglu_h=Hh)
            G.grouped_linear_dw(dy_recv, A, counts_recv, out=_mg(w_d).view(e_loc * d, inter), n_w=e_loc)
        else:
            dA = G.grouped_linear_dx(dy_recv, w_d.view(e_loc * d, inter), counts_recv, n_w=e_loc)
            G.grouped_linear_dw(dy_recv, A, counts_recv, out=_mg(w_d).view(e_loc * d, inter), n_w=e_loc)
            dH = torch.empty_like(Hh)
            ext().swiglu_bwd(dA, Hh, dH, ctx.act, counts_recv, cap)
        dxp_recv = G.grouped_linear_dx(dH, w_gu.view(e_loc * two_i, d), counts_recv, n_w=e_loc)
        G.grouped_linear_dw(dH, xp_recv, counts_recv, out=_mg(w_gu).view(e_loc * two_i, d), n_w=e_loc)
        dxp_send = _a2a(torch.empty_like(dxp_recv), dxp_recv, group)
        dh = torch.empty(ctx.t, d, dtype=torch.bfloat16, device=dev)
        ext().unpermute_add(dxp_send, sel, slot, None, dh, cap)
        ctx.w_gu = ctx.w_d = None
        return dh, dcomb, None, None, (dout if ctx.has_res else None), None, None, None, None, None


# flag purposes of the peer exchange
_DISPATCH, _Y, _DY, _DXP = 0, 1, 2, 3
_DISPATCH_B = 4  # second capacity-slot chunk of a chunked dispatch
_DY_B = 5  # second chunk of a chunked output-gradient push

# In-flight microbatch slots. A layer's receive and return buffers stay alive as saved activations
# until that microbatch's backward; a pipeline schedule with several forwards in flight (1F1B)
# gives each in-flight microbatch its own slot (``microbatch_slot``), so a later forward never
# overwrites rows an earlier microbatch's backward still reads. Every rank of an expert-parallel
# group runs the same schedule, so a slot names the same buffers on all of them.
_SLOTS = 1
_SLOT = 0


def set_inflight_microbatches(n: int) -> None:
    """Number of microbatches whose forward may run before an earlier one's backward (call before
    the first expert-parallel forward: the heap is sized from it)."""
    global _SLOTS
    _SLOTS = max(1, int(n))


class microbatch_slot:
    """``with microbatch_slot(m): forward(...)`` -- buffers of slot ``m % inflight``."""

    def __init__(self, m: int):
        self.slot = int(m) % _SLOTS

    def __enter__(self):
        global _SLOT
        self.prev, _SLOT = _SLOT, self.slot
        return self

    def __exit__(self, *exc):
        global _SLOT
        _SLOT = self.prev
        return False


def return_mode() -> str:
    """How expert outputs (forward) and input gradients (backward) travel back to their source
    ranks (``MXK_EP_RETURN``): ``pull`` (default) -- the GEMM writes locally and the source's
    combine / unpermute kernel reads the owners' rows over NVLink; ``store`` -- the grouped GEMM's
    epilogue writes them straight into the source's buffer with TMA stores into peer memory, tile by
    tile, and the source combines locally. Measured on 2 GPUs, ``store`` removes 30 ms/step of
    exposed exchange but its GEMMs (32-row x 64-byte store boxes over NVLink) slow by about as much."""
    m = os.environ.get("MXK_EP_RETURN", "pull")
    if m not in ("store", "pull"):
        raise ValueError(f"MXK_EP_RETURN must be store or pull, got {m!r}")
    return m


def _heap(group, dev, e, cap, d, n_layers):
    from .symm import heap_for, nbytes

    rows = e * cap
    # per layer and in-flight slot: the receive buffer, its counts and the return buffer
    per_layer = 2 * nbytes((rows, d), torch.bfloat16) + nbytes((e,), torch.int32) + 1024
    # shared by layers: output-gradient rows, returned input gradients, and the pull mode's buffers
    shared = 4 * nbytes((rows, d), torch.bfloat16)
    return heap_for(group, dev, per_layer * n_layers * _SLOTS + shared + (1 << 20))


# Exchange timing: while a list is installed (``exchange_timing``), every token exchange of the peer
# path records a (start, end) pair of CUDA events on the current stream around its kernels and
# waits. Nothing else runs on that stream in between, so the summed intervals are the device time
# the step spends exposed in the exchange. (Rows that travel inside a GEMM's epilogue are part of
# that GEMM's time, not of these intervals.)
_TIMING: list | None = None


class exchange_timing:
    """``with exchange_timing() as t: ...; t.ms()`` -- device milliseconds spent in token exchanges
    (dispatch, combine and their backward passes) by the code run inside the block."""

    def __enter__(self):
        global _TIMING
        self.pairs = []
        _TIMING = self.pairs
        return self

    def __exit__(self, *exc):
        global _TIMING
        _TIMING = None
        return False

    def ms(self) -> float:
        torch.cuda.synchronize()
        return float(sum(a.elapsed_time(b) for a, b in self.pairs))


def _mark():
    if _TIMING is None:
        return None
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev


def _span(start):
    if start is not None and _TIMING is not None:
        _TIMING.append((start, _mark()))


def _dispatch_chunked(h, perm, counts, heap, e_loc, cap, half, off_xp, off_cnt, xp_recv, counts_recv, w_gu2d, Hh,
                      A, dev):
    """Forward dispatch in two capacity-slot chunks overlapped with the gate/up GEMM of the first
    (``dispatch_chunks() == 2``). The comm stream pushes chunk A (slots [0, half), with the counts)
    and chunk B (slots [half, cap)) on ``comm_sms()`` CTAs, each publishing its own flag; the training
    stream, with its persistent GEMMs capped at the other SMs, waits for chunk A's flags, runs the
    SwiGLU GEMM over rows [g C, g C + min(count, half)) of every group, then waits for chunk B and
    runs it over rows [g C + half, g C + count) (the same tensors viewed ``half`` rows later)."""
    from ..ops import gemm as G
    from ..ops._ext import err_flag, ext

    my, e = heap.my, counts.numel()
    two_i, d = w_gu2d.shape[0] // e_loc, w_gu2d.shape[1]
    nblk = max(2, comm_sms())
    main = torch.cuda.current_stream(dev)
    cs = comm_stream(dev)
    ea, eb = heap.next_epoch(_DISPATCH), heap.next_epoch(_DISPATCH_B)
    cs.wait_stream(main)
    with torch.cuda.stream(cs):
        ext().ep_dispatch_push(h, perm, counts, heap.peers, my, e_loc, cap, off_xp, off_cnt, 0, _DISPATCH, ea,
                               heap.counter(_DISPATCH), 0, half, nblk)
        ext().ep_dispatch_push(h, perm, counts, heap.peers, my, e_loc, cap, off_xp, off_cnt, 0, _DISPATCH_B, eb,
                               heap.counter(_DISPATCH_B), half, 1 << 30, nblk)
    for t in (h, perm, counts):
        t.record_stream(cs)
    budget = max(2, ext().num_sms() - nblk)
    ext().set_stream_sm_budget(main.cuda_stream, budget)
    try:
        t0 = _mark()
        ext().ep_wait(heap.peers, my, 0, _DISPATCH, ea, err_flag(dev))
        _span(t0)
        cnt_a = counts_recv.clamp(max=half)
        G.gemm(xp_recv, w_gu2d, Hh, G=e, M=half, N=two_i, K=d, counts=cnt_a, ragged=1, a_grp=cap, b_grp=two_i,
               c_grp=cap, epi="swiglu", c2=A, b_mod=e_loc)
        t1 = _mark()
        ext().ep_wait(heap.peers, my, 0, _DISPATCH_B, eb, err_flag(dev))
        _span(t1)
        cnt_b = (counts_recv - half).clamp(min=0).to(torch.int32)
        G.gemm(xp_recv[half:], w_gu2d, Hh[half:], G=e, M=cap - half, N=two_i, K=d, counts=cnt_b, ragged=1,
               a_grp=cap, b_grp=two_i, c_grp=cap, epi="swiglu", c2=A[half:], b_mod=e_loc)
    finally:
        ext().set_stream_sm_budget(main.cuda_stream, 0)
    main.wait_stream(cs)


def _dy_push_chunked(dout, perm, wperm, counts, heap, e_loc, cap, half, off_dy, dy_recv, counts_recv, w_d2d, Hh,
                     dev):
    """Backward mirror of ``_dispatch_chunked``: the comm stream pushes the ``w * dout`` rows in two
    capacity-slot chunks while the training stream runs the SwiGLU-backward activation-gradient GEMM
    on the first chunk's rows; returns dH ``[rows, 2I]``."""
    from ..ops import gemm as G
    from ..ops._ext import err_flag, ext

    my, e = heap.my, counts.numel()
    d, inter = w_d2d.shape[0] // e_loc, w_d2d.shape[1]
    rows = e * cap
    nblk = max(2, comm_sms())
    main = torch.cuda.current_stream(dev)
    cs = comm_stream(dev)
    ea, eb = heap.next_epoch(_DY), heap.next_epoch(_DY_B)
    cs.wait_stream(main)
    with torch.cuda.stream(cs):
        ext().ep_combine_bwd_push(dout, perm, wperm, counts, heap.peers, my, e_loc, cap, off_dy, 0, _DY, ea,
                                  heap.counter(_DY), 0, half, nblk)
        ext().ep_combine_bwd_push(dout, perm, wperm, counts, heap.peers, my, e_loc, cap, off_dy, 0, _DY_B, eb,
                                  heap.counter(_DY_B), half, 1 << 30, nblk)
    for t in (dout, perm, wperm, counts):
        t.record_stream(cs)
    dH = torch.empty(rows, 2 * inter, dtype=torch.bfloat16, device=dev)
    ext().set_stream_sm_budget(main.cuda_stream, max(2, ext().num_sms() - nblk))
    try:
        t0 = _mark()
        ext().ep_wait(heap.peers, my, 0, _DY, ea, err_flag(dev))
        _span(t0)
        G.gemm(dy_recv, w_d2d, dH, b_mn=True, G=e, M=half, N=inter, K=d, counts=counts_recv.clamp(max=half),
               ragged=1, a_grp=cap, b_grp=d, c_grp=cap, b_mod=e_loc, epi="swiglu_bwd", r=Hh)
        t1 = _mark()
        ext().ep_wait(heap.peers, my, 0, _DY_B, eb, err_flag(dev))
        _span(t1)
        G.gemm(dy_recv[half:], w_d2d, dH[half:], b_mn=True, G=e, M=cap - half, N=inter, K=d,
               counts=(counts_recv - half).clamp(min=0).to(torch.int32), ragged=1, a_grp=cap, b_grp=d, c_grp=cap,
               b_mod=e_loc, epi="swiglu_bwd", r=Hh[half:])
    finally:
        ext().set_stream_sm_budget(main.cuda_stream, 0)
    main.wait_stream(cs)
    return dH


class _MoEEPFused(torch.autograd.Function):
    """Expert parallelism with the token exchange inside the kernels (NVLink peer memory).

    Forward: the permute kernel pushes routed rows into the owners' receive buffers; the owners'
    grouped gate/up GEMM runs on them; the down GEMM's epilogue stores each output tile straight
    into the source rank's return buffer (``return_mode() == "store"``), and after the flag wait
    the source combines its rows locally. Backward mirrors it: the combine-backward kernel pushes
    ``w * dout`` rows to the owners, and the gate/up input-gradient GEMM stores its tiles into the
    sources' buffer, which they sum locally. Per-layer buffers (receive, return) live in a
    symmetric heap and stay valid as saved activations; the output-gradient and returned
    input-gradient buffers are shared by layers (each is consumed before any peer can reach the next
    layer's exchange)."""

    @staticmethod
    def forward(ctx, h, comb, w_gu, w_d, residual, sel, keep, cap, group, act, layer, n_layers):
        from ..ops import gemm as G
        from ..ops._ext import err_flag, ext
        from ..ops.cuda_fns import _ACT, _c, dispatch_plan

        h = _c(h)
        t, d = h.shape
        e_loc, two_i, _ = w_gu.shape
        inter = two_i // 2
        world = dist.get_world_size(group)
        e = e_loc * world
        dev = h.device
        heap = _heap(group, dev, e, cap, d, n_layers)
        my = heap.my
        rows = e * cap
        key = (layer, _SLOT)
        off_xp = heap.alloc(("xp",) + key, rows * d * 2)
        off_cnt = heap.alloc(("cnt",) + key, e * 4)
        slot, perm, wperm, counts = dispatch_plan(sel, keep, comb, e, cap)
        xp_recv = heap.tensor(off_xp, (rows, d), torch.bfloat16)
        counts_recv = heap.tensor(off_cnt, (e,), torch.int32)
        Hh = torch.empty(rows, two_i, dtype=torch.bfloat16, device=dev)
        A = torch.empty(rows, inter, dtype=torch.bfloat16, device=dev)
        half = cap // 2
        if dispatch_chunks() == 2 and half % 256 == 0 and cap % 256 == 0:
            _dispatch_chunked(h, perm, counts, heap, e_loc, cap, half, off_xp, off_cnt, xp_recv, counts_recv,
                              w_gu.view(e_loc * two_i, d), Hh, A, dev)
        else:
            ep = heap.next_epoch(_DISPATCH)
            t0 = _mark()
            ext().ep_dispatch_push(h, perm, counts, heap.peers, my, e_loc, cap, off_xp, off_cnt, 0, _DISPATCH, ep,
                                   heap.counter(_DISPATCH))
            ext().ep_wait(heap.peers, my, 0, _DISPATCH, ep, err_flag(dev))
            _span(t0)
            G.grouped_linear(xp_recv, w_gu.view(e_loc * two_i, d), counts_recv, out=Hh, epi="swiglu", c2=A,
                             n_w=e_loc)
        out = torch.empty(t, d, dtype=torch.bfloat16, device=dev)
        res = None if residual is None else _c(residual)
        if return_mode() == "store":
            off_yr = heap.alloc(("yret",) + key, rows * d * 2)
            y_local = heap.tensor(off_yr, (rows, d), torch.bfloat16)  # filled by the owners' GEMMs
            G.grouped_linear(A, w_d.view(e_loc * d, inter), counts_recv, out=y_local, n_w=e_loc,
                             peer=heap.peer_store(off_yr, rows, d, e_loc, cap))
            ey = heap.next_epoch(_Y)
            t1 = _mark()
            ext().ep_signal(heap.peers, my, 0, _Y, ey)
            ext().ep_wait(heap.peers, my, 0, _Y, ey, err_flag(dev))
            ext().combine(y_local, sel, slot, _c(comb.detach().float()), res, out, cap)
            _span(t1)
        else:
            off_y = heap.alloc("y", rows * d * 2)
            y_recv = heap.tensor(off_y, (rows, d), torch.bfloat16)
            G.grouped_linear(A, w_d.view(e_loc * d, inter), counts_recv, out=y_recv, n_w=e_loc)
            ey = heap.next_epoch(_Y)
            t1 = _mark()
            ext().ep_signal(heap.peers, my, 0, _Y, ey)
            ext().ep_wait(heap.peers, my, 0, _Y, ey, err_flag(dev))
            y_local = torch.empty(rows, d, dtype=torch.bfloat16, device=dev)
            ext().ep_combine_pull(sel, slot, _c(comb.detach().float()), res, out, y_local, heap.peers, my, e_loc,
                                  cap, off_y)
            _span(t1)
        ctx.save_for_backward(xp_recv, Hh, A, y_local, sel, slot, perm, wperm, counts, counts_recv)
        ctx.w_gu, ctx.w_d, ctx.cap, ctx.act, ctx.t, ctx.heap = w_gu, w_d, cap, _ACT[act], t, heap
        ctx.has_res = residual is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        from ..ops import gemm as G
        from ..ops._ext import err_flag, ext
        from ..ops.cuda_fns import _c, _mg

        xp_recv, Hh, A, y_local, sel, slot, perm, wperm, counts, counts_recv = ctx.saved_tensors
        dout = _c(dout)
        w_gu, w_d, cap, heap = ctx.w_gu, ctx.w_d, ctx.cap, ctx.heap
        e_loc, two_i, d = w_gu.shape
        inter = two_i // 2
        dev = dout.device
        my = heap.my
        e = e_loc * heap.world
        rows = e * cap
        store = return_mode() == "store"
        off_dy = heap.alloc("dy", rows * d * 2)
        off_dxp = heap.alloc("dxret" if store else "dxp", rows * d * 2)
        dcomb = torch.empty(sel.shape, dtype=torch.float32, device=dev)
        ext().combine_bwd(dout, y_local, sel, slot, perm, wperm, counts, cap, None, dcomb)
        dy_recv = heap.tensor(off_dy, (rows, d), torch.bfloat16)
        half = cap // 2
        chunked = dispatch_chunks() == 2 and ctx.act == 0 and half % 256 == 0 and cap % 256 == 0
        if chunked:
            dH = _dy_push_chunked(dout, perm, wperm, counts, heap, e_loc, cap, half, off_dy, dy_recv, counts_recv,
                                  w_d.view(e_loc * d, inter), Hh, dev)
        else:
            edy = heap.next_epoch(_DY)
            t0 = _mark()
            ext().ep_combine_bwd_push(dout, perm, wperm, counts, heap.peers, my, e_loc, cap, off_dy, 0, _DY, edy,
                                      heap.counter(_DY))
            ext().ep_wait(heap.peers, my, 0, _DY, edy, err_flag(dev))
            _span(t0)
        # the receive buffers are reused by the next exchange: weight gradients run now, never deferred
        with G.defer_weight_grads(None):
            if ctx.act == 0:  # SiLU gate: the activation-gradient GEMM writes dH in its epilogue
                if not chunked:
                    dH = G.grouped_linear_dx(dy_recv, w_d.view(e_loc * d, inter), counts_recv, n_w=e_loc,
                                             swiglu_h=Hh)
                G.grouped_linear_dw(dy_recv, A, counts_recv, out=_mg(w_d).view(e_loc * d, inter), n_w=e_loc)
            else:
                dA = G.grouped_linear_dx(dy_recv, w_d.view(e_loc * d, inter), counts_recv, n_w=e_loc)
                G.grouped_linear_dw(dy_recv, A, counts_recv, out=_mg(w_d).view(e_loc * d, inter), n_w=e_loc)
                dH = torch.empty_like(Hh)
                ext().swiglu_bwd(dA, Hh, dH, ctx.act, counts_recv, cap)
            dxp = heap.tensor(off_dxp, (rows, d), torch.bfloat16)
            # store: each tile of input-gradient rows goes straight into its source rank's buffer
            G.grouped_linear_dx(dH, w_gu.view(e_loc * two_i, d), counts_recv, out=dxp, n_w=e_loc,
                                peer=heap.peer_store(off_dxp, rows, d, e_loc, cap) if store else None)
        exp_ = heap.next_epoch(_DXP)
        t1 = _mark()
        ext().ep_signal(heap.peers, my, 0, _DXP, exp_)
        _span(t1)
        # The gate/up weight gradient reads dH (local) and this layer's own receive buffer, never the
        # shared dy / returned-gradient buffers, so it runs while the input-gradient rows travel.
        with G.defer_weight_grads(None):
            G.grouped_linear_dw(dH, xp_recv, counts_recv, out=_mg(w_gu).view(e_loc * two_i, d), n_w=e_loc)
        t2 = _mark()
        ext().ep_wait(heap.peers, my, 0, _DXP, exp_, err_flag(dev))
        dh = torch.empty(ctx.t, d, dtype=torch.bfloat16, device=dev)
        if store:
            ext().unpermute_add(dxp, sel, slot, None, dh, cap)
        else:
            ext().ep_unpermute_pull(sel, slot, dh, heap.peers, my, e_loc, cap, off_dxp)
        _span(t2)
        ctx.w_gu = ctx.w_d = ctx.heap = None
        return (dh, dcomb, None, None, (dout if ctx.has_res else None), None, None, None, None, None, None, None)


def _moe_ep_cpu(h, r, w_gu, w_d, cap, group, residual, act):
    """Differentiable CPU/gloo version (torch ops + autograd all-to-all); the oracle of the GPU path."""
    from torch.distributed.nn.functional import all_to_all_single

    from ..ops import reference as R
    from ..ops.layout import split_gate_up

    t, d = h.shape
    e_loc = w_gu.shape[0]
    inter = w_d.shape[2]
    world = dist.get_world_size(group)
    e = e_loc * world
    keep = None if bool(r.keep.all()) else r.keep
    slots, counts = R.capacity_slots(r.selected, e, cap, keep)
    valid = slots >= 0
    rows = (r.selected * cap + slots.clamp_min(0))[valid]
    tok = torch.arange(t).unsqueeze(1).expand_as(r.selected)[valid]
    send = torch.zeros(e * cap, d, dtype=h.dtype)
    send = send.index_copy(0, rows, h[tok])
    cnt_recv = torch.empty_like(counts)
    dist.all_to_all_single(cnt_recv, counts.contiguous(), group=group)
    recv = all_to_all_single(torch.empty_like(send), send, group=group)
    outs = []
    for g in range(world * e_loc):
        ex = g % e_loc
        xg = recv[g * cap:(g + 1) * cap]
        hg = xg @ w_gu[ex].t()
        gg, uu = split_gate_up(hg, inter)
        outs.append((R.activation(gg, act) * uu) @ w_d[ex].t())
    y_recv = torch.cat(outs, 0)
    y_send = all_to_all_single(torch.empty_like(y_recv), y_recv, group=group)
    w = (r.combine * valid.to(r.combine.dtype))[valid]
    contrib = y_send[rows] * w.unsqueeze(1).to(y_send.dtype)
    out = torch.zeros(t, d, dtype=h.dtype).index_add(0, tok, contrib)
    return out if residual is None else residual + out


# ------------------------------------------------------------------ shared expert beside the exchange
# Under the peer-memory exchange much of the MoE layer's device time is the token exchanges (NVLink
# transfers inside the push / pull kernels and the waits for the slowest peer), which a single
# stream cannot overlap with compute. The shared expert depends only on the layer input, so it can
# run on a side stream meanwhile, forward and (through autograd's per-stream backward) backward.
# The side stream's persistent GEMMs are capped at all but comm_sms() SMs, so the exchange kernels
# keep SMs beside them. On by default (MXK_EP_OVERLAP=0 turns it off): the megagpt step's
# ms x median-MHz was 3-4 % lower with it on 2 GPUs and 7 % lower on 8 (1.163e6 vs 1.256e6).
_SIDE: dict[int, torch.cuda.Stream] = {}


def overlap_shared_enabled(h: torch.Tensor, group) -> bool:
    """Shared expert on a side stream: CUDA tensors, an expert-parallel group, the peer-memory
    exchange, and ``MXK_EP_OVERLAP`` not set to 0."""
    return (h.is_cuda and group is not None and ep_impl() == "peer"
            and os.environ.get("MXK_EP_OVERLAP", "1") == "1")


def dispatch_chunks() -> int:
    """Forward dispatch in capacity-slot chunks (``MXK_EP_CHUNKS``: 1, the default, or 2). With 2, a
    comm stream pushes slots [0, C/2) and then [C/2, C) of every expert on ``comm_sms()`` CTAs while
    the training stream, capped at the remaining SMs, waits for the first chunk's flags and runs the
    gate/up GEMM on those rows as the second chunk crosses NVLink."""
    n = int(os.environ.get("MXK_EP_CHUNKS", "1"))
    if n not in (1, 2):
        raise ValueError(f"MXK_EP_CHUNKS must be 1 or 2, got {n}")
    return n


_COMM: dict[int, torch.cuda.Stream] = {}


def comm_stream(dev: torch.device) -> torch.cuda.Stream:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    s = _COMM.get(idx)
    if s is None:
        s = _COMM[idx] = torch.cuda.Stream(device=torch.device("cuda", idx))
    return s


def comm_sms() -> int:
    """SMs that side-stream GEMMs leave free for the exchange kernels (``MXK_EP_COMM_SMS``, default 16;
    even, so CTA-pair GEMM tiles keep whole pairs)."""
    n = int(os.environ.get("MXK_EP_COMM_SMS", "16"))
    return max(0, n + (n & 1))


def side_stream(dev: torch.device) -> torch.cuda.Stream:
    """The device's side stream; persistent GEMMs launched on it use all but ``comm_sms()`` SMs."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    s = _SIDE.get(idx)
    if s is None:
        from ..ops._ext import ext

        s = _SIDE[idx] = torch.cuda.Stream(device=torch.device("cuda", idx))
        reserve = comm_sms()
        if reserve > 0:
            ext().set_stream_sm_budget(s.cuda_stream, max(2, ext().num_sms() - reserve))
    return s


class _JoinShared(torch.autograd.Function):
    """``y + s`` where ``s`` (the shared expert's output) was computed on the side stream.

    Forward: the training stream waits for the side stream, then adds. Backward: both inputs get the
    incoming gradient; the side stream uses it (``record_stream`` keeps its memory from being reused
    meanwhile). The shared expert's backward writes its weight gradients into ``main_grad`` outside
    autograd, so a callback at the end of the backward pass makes the training stream wait for the
    side stream: whatever reads the gradients next (all-reduce, optimizer) sees them complete."""

    @staticmethod
    def forward(ctx, y, s, side, main):
        main.wait_stream(side)
        s.record_stream(main)
        ctx.side, ctx.main = side, main
        return y + s

    @staticmethod
    def backward(ctx, g):
        side, main = ctx.side, ctx.main
        g.record_stream(side)
        torch.autograd.Variable._execution_engine.queue_callback(lambda: main.wait_stream(side))
        ctx.side = ctx.main = None
        return g, g, None, None


def with_shared_overlap(h: torch.Tensor, shared_fn, moe_fn):
    """``moe_fn()`` (returning ``(y, extra)``, y without the shared expert) on the current stream
    while ``shared_fn(h)`` runs on the side stream; returns ``(y + shared_fn(h), extra)``."""
    main = torch.cuda.current_stream(h.device)
    side = side_stream(h.device)
    side.wait_stream(main)
    h.record_stream(side)
    with torch.cuda.stream(side):
        s = shared_fn(h)
    y, extra = moe_fn()
    return _JoinShared.apply(y, s, side, main), extra


def ep_impl() -> str:
    """``peer`` (default on GPUs): exchange inside the kernels over NVLink peer memory;
    ``nccl``: the same capacity layout moved by NCCL all-to-alls (the baseline path)."""
    return os.environ.get("MXK_EP_IMPL", "peer")


def moe_experts_ep(h, r, w_gate_up, w_down, capacity, group, residual=None, act: str = "silu", layer: int = 0,
                   n_layers: int = 1):
    t = h.shape[0]
    cap = capacity if capacity is not None else ops.capacity_for(t, r.selected.shape[1], 1, 1.0)
    if not h.is_cuda:
        return _moe_ep_cpu(h, r, w_gate_up, w_down, cap, group, residual, act)
    keep = None if r.keep is None else r.keep.to(torch.uint8)
    if ep_impl() == "peer" and dist.get_world_size(group) <= 16:
        return _MoEEPFused.apply(h, r.combine, w_gate_up, w_down, residual, r.selected, keep, cap, group, act, layer,
                                 n_layers)
    return _MoEEP.apply(h, r.combine, w_gate_up, w_down, residual, r.selected, keep, cap, group, act)
