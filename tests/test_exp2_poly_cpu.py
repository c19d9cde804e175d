"""The FMA-pipe exp2 used for part of the attention softmax (``ex2_poly2`` in
``ops/csrc/sm100_primitives.cuh``), emulated bit-exactly in float32 with numpy: range reduction by
the 1.5 * 2^23 shifter, degree-3 polynomial for 2^f on [-1/2, 1/2], exponent-field scaling, clamp at
-126. Checks the relative error bound, and that very negative and -inf arguments give ~0 (never a
negative number or NaN from a borrow into the sign bit)."""

import os
import re

import numpy as np

HDR = os.path.join(os.path.dirname(__file__), "..", "marin_experiments_b200", "ops", "csrc", "sm100_primitives.cuh")


def _coeffs():
    src = open(HDR).read()
    body = src[src.index("void ex2_poly2("):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"f2_make\(([0-9.]+)f, \1f\)", body) if float(v) < 2.0]
    c3, c2, c1, c0 = vals[:4]  # q = c3 f + c2; q = q f + c1; q = q f + c0
    return np.float32(c3), np.float32(c2), np.float32(c1), np.float32(c0)


def _ex2_poly(x):
    c3, c2, c1, c0 = _coeffs()
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    f = (x - j).astype(np.float32)
    q = (c3 * f + c2).astype(np.float32)
    q = (q * f + c1).astype(np.float32)
    q = (q * f + c0).astype(np.float32)
    bits = (q.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_exp2_poly_accuracy_and_range():
    x = np.concatenate([np.linspace(-40.0, 0.0, 200001, dtype=np.float32),
                        np.array([-np.inf, -1e30, -200.0, -126.6, -126.4, -126.0, -125.5, 0.0], np.float32)])
    y = _ex2_poly(x)
    assert np.isfinite(y).all() and (y >= 0).all()
    ref = np.exp2(np.maximum(x.astype(np.float64), -1000.0))
    big = ref > 1e-30
    assert np.max(np.abs(y[big] - ref[big]) / ref[big]) < 1e-4  # bf16 half-ulp is 2^-9 ~ 2e-3
    assert np.max(y[~big]) < 1e-37
