"""The allocation-free C entry point of the dispatch plan (``mxk_dispatch_plan_noalloc``).

Called through its exported C symbol with ctypes, the way a caller that cannot allocate device
memory would call it (inputs and outputs preallocated, scratch inside the library), and compared
with the regular dispatch-plan op on two calls in a row.
"""

import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    from marin_experiments_b200.ops._ext import ext
    from marin_experiments_b200.ops.build import BUILD_DIR, EXT_NAME

    ext()  # the library (and its torch dependencies) is loaded by the package first
    lib = ctypes.CDLL(os.path.join(BUILD_DIR, EXT_NAME + ".so"))
    f = lib.mxk_dispatch_plan_noalloc
    f.restype = ctypes.c_int
    vp = ctypes.c_void_p
    f.argtypes = [vp, vp, vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, vp, vp, vp, vp, vp]
    return f


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


@pytest.mark.parametrize("e", [64, 512, 1024])
def test_noalloc_dispatch_plan_matches_op(e):
    from marin_experiments_b200.ops import cuda_fns

    f = _entry()
    t, k, cap = 6000, 4, 384
    gen = torch.Generator().manual_seed(0)
    for call in range(2):
        sel = torch.randint(0, e, (t, k), generator=gen).int().cuda()
        keep = (torch.rand(t, k, generator=gen) > 0.1).to(torch.uint8).cuda()
        comb = torch.rand(t, k, generator=gen).cuda()
        ref_slot, ref_perm, ref_wperm, ref_counts = cuda_fns.dispatch_plan(sel, keep, comb, e, cap)
        slot = torch.full((t, k), -7, dtype=torch.int32, device="cuda")
        perm = torch.zeros(e * cap, dtype=torch.int32, device="cuda")
        wperm = torch.zeros(e * cap, dtype=torch.float32, device="cuda")
        counts = torch.zeros(e, dtype=torch.int32, device="cuda")
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = f(_ptr(sel), _ptr(keep), _ptr(comb), t, k, e, cap, _ptr(slot), _ptr(perm), _ptr(wperm), _ptr(counts),
               stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: rc={rc}"
        assert torch.equal(slot, ref_slot)
        assert torch.equal(counts, ref_counts)
        for ei in range(e):
            c = int(counts[ei])
            s = slice(ei * cap, ei * cap + c)
            assert torch.equal(perm[s], ref_perm[s])
            assert torch.allclose(wperm[s], ref_wperm[s], rtol=0, atol=0)


def test_noalloc_rejects_oversized_problem():
    f = _entry()
    t, k, e = 1 << 20, 8, 512  # ceil(t*k/4096) * e far beyond the scratch array
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = f(_ptr(dummy), _ptr(None), _ptr(dummy), t, k, e, 128, _ptr(dummy), _ptr(dummy), _ptr(dummy), _ptr(dummy),
           stream)
    assert rc == 1  # MXK_NOALLOC_TOO_LARGE, nothing launched


def test_noalloc_rejects_too_many_experts():
    f = _entry()
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = f(_ptr(dummy), _ptr(None), _ptr(dummy), 4, 1, 1025, 128, _ptr(dummy), _ptr(dummy), _ptr(dummy), _ptr(dummy),
           stream)
    assert rc == 1  # MXK_NOALLOC_TOO_LARGE: above the 1024-expert limit, nothing launched
