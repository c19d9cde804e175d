"""sm_100a tcgen05 GEMM vs a plain fp32 PyTorch reference (every layout, epilogue and grouping)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.fixture(scope="module")
def G():
    from marin_experiments_b200.ops import gemm

    return gemm


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (384, 1536, 1536), (200, 128, 320),
                                   (1024, 64, 1536), (512, 6144, 1536)])
def test_linear_fwd(G, m, n, k):
    x, w = _rand(m, k), _rand(n, k)
    y = G.linear(x, w)
    ref = x.float() @ w.float().t()
    torch.cuda.synchronize()
    assert _rel(y, ref) < 1e-2


@pytest.mark.parametrize("m,n,k", [(256, 256, 128), (512, 1536, 768), (384, 128, 256)])
def test_linear_dx(G, m, n, k):
    dy, w = _rand(m, n), _rand(n, k)
    dx = G.linear_dx(dy, w)
    assert _rel(dx, dy.float() @ w.float()) < 1e-2


@pytest.mark.parametrize("t,n,k", [(256, 256, 128), (1024, 1536, 768), (320, 128, 256)])
def test_linear_dw_accum(G, t, n, k):
    dy, x = _rand(t, n), _rand(t, k)
    base = torch.randn(n, k, device="cuda")
    out = base.clone()
    G.linear_dw(dy, x, out=out, accum=True)
    ref = base + dy.float().t() @ x.float()
    assert _rel(out, ref) < 1e-3


def test_grouped_ragged_fwd_dx_dw(G):
    torch.manual_seed(0)
    g, cap, d, n = 8, 384, 256, 512
    counts = torch.tensor([0, 5, 128, 129, 384, 250, 64, 300], dtype=torch.int32, device="cuda")
    x = _rand(g * cap, d)
    for e in range(g):  # zero the pad rows (the capacity-layout invariant)
        x[e * cap + counts[e]:(e + 1) * cap] = 0
    w = _rand(g * n, d)
    y = torch.full((g * cap, n), 7.0, dtype=torch.bfloat16, device="cuda")
    G.grouped_linear(x, w, counts, out=y)
    dy = _rand(g * cap, n)
    for e in range(g):
        dy[e * cap + counts[e]:(e + 1) * cap] = 0
    dx = G.grouped_linear_dx(dy, w, counts)
    dw = torch.zeros(g * n, d, device="cuda")
    G.grouped_linear_dw(dy, x, counts, out=dw)
    torch.cuda.synchronize()
    for e in range(g):
        c = int(counts[e])
        xs, ws, dys = x[e * cap:e * cap + c].float(), w[e * n:(e + 1) * n].float(), dy[e * cap:e * cap + c].float()
        if c:
            assert _rel(y[e * cap:e * cap + c], xs @ ws.t()) < 1e-2
            assert _rel(dx[e * cap:e * cap + c], dys @ ws) < 1e-2
            assert _rel(dw[e * n:(e + 1) * n], dys.t() @ xs) < 1e-2
        else:
            assert (dw[e * n:(e + 1) * n] == 0).all()


@pytest.mark.parametrize("g", [257, 1024])
def test_grouped_many_groups(G, g):
    """More groups than prefix-table slots (256): tiles are decoded through a slot's group walk."""
    torch.manual_seed(1)
    cap, d, n = 128, 128, 256
    counts = torch.randint(0, cap + 1, (g,), dtype=torch.int32)
    counts[::7] = 0  # empty groups inside and across slots
    counts = counts.cuda()
    x = _rand(g * cap, d)
    rows = torch.arange(g * cap, device="cuda") % cap
    x[rows >= counts.repeat_interleave(cap)] = 0
    w = _rand(g * n, d)
    y = torch.zeros(g * cap, n, dtype=torch.bfloat16, device="cuda")
    G.grouped_linear(x, w, counts, out=y)
    torch.cuda.synchronize()
    ref = torch.einsum("gck,gnk->gcn", x.view(g, cap, d).float(), w.view(g, n, d).float()).reshape(g * cap, n)
    valid = (rows < counts.repeat_interleave(cap)).unsqueeze(1)
    assert _rel(y.float() * valid, ref * valid) < 1e-2


def test_swiglu_epilogue(G):
    m, d, inter = 256, 256, 512
    x = _rand(m, d)
    w = _rand(2 * inter, d, scale=0.1)  # blocked layout: [gate 128 | up 128] per 256 rows
    h = torch.empty(m, 2 * inter, dtype=torch.bfloat16, device="cuda")
    a = torch.empty(m, inter, dtype=torch.bfloat16, device="cuda")
    G.linear(x, w, out=h, epi="swiglu", c2=a)
    hr = x.float() @ w.float().t()
    hb = hr.view(m, inter // 128, 2, 128)
    ar = (F.silu(hb[:, :, 0]) * hb[:, :, 1]).reshape(m, inter)
    assert _rel(h, hr) < 1e-2
    assert _rel(a, ar) < 2e-2


def test_resid_gate_silu_epilogues(G):
    m, k, n = 256, 128, 256
    x, w, r = _rand(m, k), _rand(n, k, scale=0.1), _rand(m, n)
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    G.linear(x, w, out=out, epi="resid", r=r)
    assert _rel(out, x.float() @ w.float().t() + r.float()) < 1e-2
    G.linear(x, w, out=out, epi="gate_mul", r=r)
    assert _rel(out, r.float() * torch.sigmoid(x.float() @ w.float().t())) < 1e-2
    w2 = _rand(128, k, scale=0.1)
    s = torch.empty(m, 128, dtype=torch.bfloat16, device="cuda")
    hh = torch.empty(m, 128, dtype=torch.bfloat16, device="cuda")
    G.linear(x, w2, out=s, epi="silu", c2=hh)
    assert _rel(s, F.silu(x.float() @ w2.float().t())) < 2e-2


def test_ce_epilogue(G):
    m, k, v = 256, 128, 1000  # vocab not a multiple of the tile
    h, w = _rand(m, k), _rand(v, k, scale=0.5)
    nt = (v + 255) // 256
    vpad = nt * 256
    logits = torch.empty(m, vpad, dtype=torch.bfloat16, device="cuda")
    stats = torch.empty(m, 2 * nt, 2, dtype=torch.float32, device="cuda")  # one entry per tile half
    G.gemm(h, w, logits, M=m, N=v, K=k, epi="ce", c2=stats.view(m, nt * 4))
    ref = h.float() @ w.float().t()
    assert _rel(logits[:, :v], ref) < 1e-2
    mx, se = stats[..., 0], stats[..., 1]
    gmax = mx.max(1, keepdim=True).values
    lse = gmax.squeeze(1) + torch.log((se * torch.exp(mx - gmax)).sum(1))
    assert torch.allclose(lse, torch.logsumexp(ref, 1), atol=5e-2, rtol=1e-3)


def test_deferred_weight_grads_match():
    """Zero-bubble B/W split: inside defer_weight_grads the weight-gradient GEMMs are queued, the
    input gradient is complete, and running the queue later gives the same main_grad."""
    from marin_experiments_b200.ops import cuda_fns
    from marin_experiments_b200.ops import gemm as G

    torch.manual_seed(0)
    x = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.nn.Parameter(torch.randn(384, 512, device="cuda", dtype=torch.bfloat16) / 16)
    w.main_grad = torch.zeros(384, 512, device="cuda")
    g = torch.randn(256, 384, device="cuda", dtype=torch.bfloat16)
    xa = x.clone().requires_grad_(True)
    cuda_fns.linear(xa, w).backward(g)
    ref_dx, ref_dw = xa.grad.clone(), w.main_grad.clone()
    w.main_grad.zero_()
    xb = x.clone().requires_grad_(True)
    q = []
    with G.defer_weight_grads(q):
        cuda_fns.linear(xb, w).backward(g)
    assert len(q) == 1 and float(w.main_grad.abs().sum()) == 0.0
    assert torch.equal(xb.grad, ref_dx)
    G.run_weight_grads(q)
    # split-K partial sums are combined with atomic adds: equal up to summation order
    assert torch.allclose(w.main_grad, ref_dw, rtol=1e-4, atol=1e-3)


def test_pair_tile_shapes(G):
    """Shapes that take the CTA-pair (256-row) tiles: grouped problems whose per-group rows are a
    multiple of 256 (ragged counts inside), a row count that leaves the second CTA of the last
    pair out of range, and the residual / gate epilogues."""
    torch.manual_seed(3)
    g, cap, d, n = 4, 512, 256, 768
    counts = torch.tensor([512, 3, 260, 0], dtype=torch.int32, device="cuda")
    x = _rand(g * cap, d)
    for e in range(g):
        x[e * cap + counts[e]:(e + 1) * cap] = 0
    w = _rand(g * n, d)
    y = G.grouped_linear(x, w, counts)
    dy = _rand(g * cap, n)
    for e in range(g):
        dy[e * cap + counts[e]:(e + 1) * cap] = 0
    dx = G.grouped_linear_dx(dy, w, counts)
    torch.cuda.synchronize()
    for e in range(g):
        c = int(counts[e])
        if c:
            xs, ws, dys = x[e * cap:e * cap + c].float(), w[e * n:(e + 1) * n].float(), dy[e * cap:e * cap + c].float()
            assert _rel(y[e * cap:e * cap + c], xs @ ws.t()) < 1e-2
            assert _rel(dx[e * cap:e * cap + c], dys @ ws) < 1e-2
    m, k, n = 384, 512, 1536
    a, b, r = _rand(m, k), _rand(n, k, scale=0.1), _rand(m, n)
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    G.linear(a, b, out=out, epi="resid", r=r)
    assert _rel(out, r.float() + a.float() @ b.float().t()) < 1e-2
    G.linear(a, b, out=out, epi="gate_mul", r=r)
    assert _rel(out, r.float() * torch.sigmoid(a.float() @ b.float().t())) < 1e-2
    base = torch.randn(n, k, device="cuda")
    acc = base.clone()
    G.linear_dw(_rand(m, n), a, out=acc, accum=True)  # 1536-row output, split over K
    torch.cuda.synchronize()


def _swiglu_bwd_ref(dA, H):
    m, inter = dA.shape
    hb = H.float().view(m, inter // 128, 2, 128)
    g, u = hb[:, :, 0], hb[:, :, 1]
    d = dA.float().view(m, inter // 128, 128)
    s = torch.sigmoid(g)
    dg = d * u * s * (1 + g * (1 - s))
    du = d * g * s
    return torch.stack([dg, du], 2).reshape(m, 2 * inter)


def test_swiglu_bwd_epilogue(G):
    """Activation-gradient GEMM whose epilogue writes the SwiGLU gate/up gradients directly
    (dense: single-CTA and pair tiles; grouped ragged-M over a capacity layout)."""
    torch.manual_seed(4)
    for m in (128, 384):
        d, inter = 256, 512
        dy, w = _rand(m, d), _rand(d, inter, scale=0.1)
        H = _rand(m, 2 * inter)
        dH = G.linear_dx(dy, w, swiglu_h=H)
        ref = _swiglu_bwd_ref(dy.float() @ w.float(), H)
        assert _rel(dH, ref) < 2e-2
    g, cap, d, inter = 4, 512, 256, 768
    counts = torch.tensor([512, 3, 260, 0], dtype=torch.int32, device="cuda")
    dy = _rand(g * cap, d)
    for e in range(g):
        dy[e * cap + counts[e]:(e + 1) * cap] = 0
    w = _rand(g * d, inter, scale=0.1)
    H = _rand(g * cap, 2 * inter)
    dH = G.grouped_linear_dx(dy, w, counts, swiglu_h=H)
    torch.cuda.synchronize()
    for e in range(g):
        c = int(counts[e])
        if c:
            r = slice(e * cap, e * cap + c)
            ref = _swiglu_bwd_ref(dy[r].float() @ w[e * d:(e + 1) * d].float(), H[r])
            assert _rel(dH[r], ref) < 2e-2
    # more tiles than workers (the epilogue's H loads run ahead across tiles) and N = 384, whose last
    # tile has an activation block past N: pair tiles, dense
    m, d, inter = 16384, 256, 384
    dy, w = _rand(m, d), _rand(d, inter, scale=0.1)
    H = _rand(m, 2 * inter)
    dH = G.linear_dx(dy, w, swiglu_h=H)
    assert _rel(dH, _swiglu_bwd_ref(dy.float() @ w.float(), H)) < 2e-2
    # single-CTA tiles (capacity 384 is not a multiple of 256), 288 tiles, grouped
    g, cap, d, inter = 16, 384, 256, 1536
    counts = torch.randint(200, cap + 1, (g,), dtype=torch.int32, device="cuda")
    dy = _rand(g * cap, d)
    for e in range(g):
        dy[e * cap + counts[e]:(e + 1) * cap] = 0
    w = _rand(g * d, inter, scale=0.1)
    H = _rand(g * cap, 2 * inter)
    dH = G.grouped_linear_dx(dy, w, counts, swiglu_h=H)
    for e in range(g):
        r = slice(e * cap, e * cap + int(counts[e]))
        ref = _swiglu_bwd_ref(dy[r].float() @ w[e * d:(e + 1) * d].float(), H[r])
        assert _rel(dH[r], ref) < 2e-2
