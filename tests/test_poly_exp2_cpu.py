"""The FMA-pipe exp2 used for part of the streamed exponentials
(poly_exp2x2 in csrc/gr_device.cuh), restated step by step in float32 with the
coefficients read from the source: relative error against 2**t within 4e-7 on
the range the streamed sums use, overflow to inf/NaN at t >= 128, NaN kept."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(__file__), "..", "vllm_gr_ehaleva_b200", "csrc", "gr_device.cuh")


def _coeffs():
    text = open(SRC).read()
    c = {k: float(v) for k, v in re.findall(r"(kP\d) = ([0-9.eE+-]+)f", text)}
    return [np.float32(c[f"kP{i}"]) for i in range(6)]


def _fma(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def poly_exp2(t):
    p0, p1, p2, p3, p4, p5 = _coeffs()
    t = np.asarray(t, np.float32)
    nan = np.isnan(t)
    t = np.minimum(np.maximum(np.where(nan, 0, t), np.float32(-125)), np.float32(128)).astype(np.float32)
    magic = np.float32(12582912.0)
    r = (t + magic).astype(np.float32)
    n = (r - magic).astype(np.float32)
    f = _fma(n, np.full_like(n, -1), t)
    p = _fma(np.full_like(f, p5), f, np.full_like(f, p4))
    for c in (p3, p2, p1, p0):
        p = _fma(p, f, np.full_like(f, c))
    bits = (r.view(np.uint32).astype(np.uint64) * 0x800000 + p.view(np.uint32).astype(np.uint64)) & 0xFFFFFFFF
    out = bits.astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), out)


def test_relative_error_on_the_streamed_range():
    rng = np.random.default_rng(0)
    t = np.concatenate([np.linspace(-120, 127, 2_000_001, dtype=np.float32),
                        rng.uniform(-30, 5, 1_000_000).astype(np.float32)])
    got = poly_exp2(t).astype(np.float64)
    ref = np.exp2(t.astype(np.float64))
    rel = np.abs(got / ref - 1)
    assert rel.max() < 4e-7, rel.max()


def test_edges():
    assert np.all(~np.isfinite(poly_exp2(np.array([128.0, 200.0, np.inf], np.float32))))
    tiny = poly_exp2(np.array([-126.0, -1000.0, -np.inf], np.float32))
    assert np.all(tiny > 0) and np.all(tiny < 1e-37)
    assert np.isnan(poly_exp2(np.array([np.nan], np.float32)))[0]
    assert poly_exp2(np.array([0.0], np.float32))[0] == np.float32(1.0) or \
        abs(float(poly_exp2(np.array([0.0], np.float32))[0]) - 1) < 2e-7
