"""The softmax's FMA-pipe exp2 (ex2_poly2 in tc_ptx.cuh), restated in numpy float32
with the constants read from the header: relative error far below a bf16 half-ulp
(P is rounded to bf16 right after) over the range the softmax feeds it."""
import re

import numpy as np

from conftest import ROOT

HEADER = (ROOT / 'dynamic-kv-cache_b200' / 'csrc' / 'tc_ptx.cuh').read_text()


def _coeffs():
    body = HEADER[HEADER.index('ex2_poly2'):]
    body = body[:body.index('return')]
    hexes = re.findall(r'(0x1\.[0-9a-f]+p-\d+)f', body)[::2]  # each constant appears twice (x, y)
    return [np.float32(float.fromhex(h)) for h in hexes]     # c3, c2, c1, c0 (Horner order)


def ex2_poly(x):
    c3, c2, c1, c0 = _coeffs()
    x = np.maximum(x.astype(np.float32), np.float32(-126.5))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    f = (x - j).astype(np.float32)
    p = (((c3 * f + c2) * f + c1) * f + c0).astype(np.float32)
    bits = (p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_polynomial_exp2_error_bound():
    assert len(_coeffs()) == 4
    x = np.concatenate([np.linspace(-125, 8, 1_000_001), -np.random.default_rng(0).random(100_000) * 40])
    x = x.astype(np.float32)
    rel = np.abs(ex2_poly(x).astype(np.float64) / np.exp2(x.astype(np.float64)) - 1)
    assert rel.max() < 1e-4 < 2.0 ** -9


def test_polynomial_exp2_tiny_below_range():
    out = ex2_poly(np.array([-200.0, -np.inf, -126.9], np.float32))
    assert np.all(out >= 0) and np.all(out < 1e-37)
