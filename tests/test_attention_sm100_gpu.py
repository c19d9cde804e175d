"""tcgen05 flash-attention forward vs the fp32 oracle (and the mma.sync kernel)."""

import math

import pytest
import torch

from marin_experiments_b200.ops import reference as R

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("hd,h,hkv,s,window,segs", [
    (64, 4, 4, 256, 0, False),
    (96, 4, 2, 512, 0, False),
    (96, 2, 2, 384, 200, False),
    (128, 2, 1, 256, 0, True),
    (96, 4, 4, 200, 0, False),
    (96, 2, 2, 2048, 0, False),  # the benchmark model's sequence length and head size
])
def test_fa_fwd_sm100(hd, h, hkv, s, window, segs):
    from marin_experiments_b200.ops._ext import check_kernel_errors, err_flag, ext

    torch.manual_seed(0)
    b = 2
    t = b * s
    q = torch.randn(t, h, hd, device="cuda").bfloat16()
    k = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    # v as a strided view inside a wider row (the fused qkv layout)
    wide = torch.randn(t, 3 * hkv * hd + 64, device="cuda").bfloat16()
    v = wide[:, hkv * hd: 2 * hkv * hd].view(t, hkv, hd)
    seg = ((torch.arange(s) // 100).repeat(b).int().cuda()) if segs else None
    o = torch.empty(t, h, hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(t, h, device="cuda")
    scale = 1 / math.sqrt(hd)
    ext().flash_fwd_sm100(q, k, v, o, lse, seg, b, s, window, scale, err_flag(q.device), None)
    torch.cuda.synchronize()
    check_kernel_errors()
    ref = R.attention(q.view(b, s, h, hd).float(), k.view(b, s, hkv, hd).float(), v.reshape(b, s, hkv, hd).float(),
                      window=window, segment_ids=None if seg is None else seg.view(b, s))
    assert rel(o.view(b, s, h, hd), ref) < 1e-2
    o2 = torch.empty_like(o)
    lse2 = torch.empty_like(lse)
    ext().flash_fwd(q, k, v, o2, lse2, seg, b, s, window, scale)
    assert torch.allclose(lse, lse2, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("hd,h,hkv,s,window,segs,acc", [
    (64, 4, 4, 256, 0, False, False),
    (96, 4, 2, 512, 0, False, True),
    (96, 2, 2, 384, 200, False, False),
    (128, 2, 1, 256, 0, True, False),
    (96, 4, 4, 200, 0, False, True),
    (96, 2, 2, 2048, 0, False, False),  # the benchmark model's sequence length and head size
])
def test_fa_bwd_sm100(hd, h, hkv, s, window, segs, acc):
    """tcgen05 backward vs the fp32 oracle's autograd gradients (and dV accumulation into an
    existing buffer, as the fused qkv gradient uses it)."""
    from marin_experiments_b200.ops._ext import check_kernel_errors, err_flag, ext

    torch.manual_seed(1)
    b = 2
    t = b * s
    q = torch.randn(t, h, hd, device="cuda").bfloat16()
    k = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    v = torch.randn(t, hkv, hd, device="cuda").bfloat16()
    seg = ((torch.arange(s) // 100).repeat(b).int().cuda()) if segs else None
    o = torch.empty(t, h, hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(t, h, device="cuda")
    scale = 1 / math.sqrt(hd)
    ext().flash_fwd_sm100(q, k, v, o, lse, seg, b, s, window, scale, err_flag(q.device), None)
    do = torch.randn(t, h, hd, device="cuda").bfloat16()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv0 = torch.randn(t, hkv, hd, device="cuda").bfloat16() if acc else torch.zeros(t, hkv, hd, device="cuda").bfloat16()
    dv = dv0.clone()
    dqa = torch.empty(t, h, hd, device="cuda")
    dsum = torch.empty(t, h, device="cuda")
    ext().flash_bwd_sm100(q, k, v, o, lse, seg, b, s, window, scale, do, dsum, dqa, dq, dk, dv, acc, err_flag(q.device))
    torch.cuda.synchronize()
    check_kernel_errors()
    qf = q.view(b, s, h, hd).float().requires_grad_(True)
    kf = k.view(b, s, hkv, hd).float().requires_grad_(True)
    vf = v.view(b, s, hkv, hd).float().requires_grad_(True)
    ref = R.attention(qf, kf, vf, window=window, segment_ids=None if seg is None else seg.view(b, s))
    ref.backward(do.view(b, s, h, hd).float())
    assert rel(dq.view(b, s, h, hd), qf.grad) < 2e-2
    assert rel(dk.view(b, s, hkv, hd), kf.grad) < 2e-2
    want_dv = vf.grad + (dv0.view(b, s, hkv, hd).float() if acc else 0)
    assert rel(dv.view(b, s, hkv, hd), want_dv) < 2e-2
