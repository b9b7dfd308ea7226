"""The oracle's config-3 epilogue (BitLinear output -> BitShift norm ->
ste_clamp + squareplus, statistics from the exact integer row sums) against
the same definition composed here from numpy (float64 statistics of exact
int64 sums, fp32 elementwise products) and the oracle's squareplus stage,
which the golden fixtures pin to the reference."""
from fractions import Fraction

import numpy as np
import pytest

from oracle import lib as orc

_THRESH = [(4.0, 0.5), (16.0, 0.25), (64.0, 0.125), (256.0, 0.0625), (1024.0, 0.03125), (4096.0, 0.015625),
           (16384.0, 0.0078125), (65536.0, 0.00390625)]


def _pow2(v: float) -> np.float32:
    # _find_power_of_2_scale's table (src/mamba_integer_model.py:144-184)
    s = 1.0
    for t, sc in _THRESH:
        if v >= t:
            s = sc
    if v < 1.0:
        s = 1.0
    if v < 0.25:
        s = 2.0
    if v < 0.0625:
        s = 4.0
    if v < 0.015625:
        s = 8.0
    return np.float32(s)


def _composed(acc, a_scale, w_scale, gamma, step):
    M, N = acc.shape
    out = np.empty((M, N), np.float32)
    for m in range(M):
        r = acc[m].astype(np.int64)
        s1, s2 = int(r.sum()), int((r * r).sum())
        sc = np.float32(np.float32(w_scale) * np.float32(a_scale[m]))
        dsc = np.float64(sc)
        mean = np.float32((np.float64(s1) / np.float64(N)) * dsc)
        vnum = N * s2 - s1 * s1
        assert vnum == int(Fraction(N * s2 - s1 * s1))  # exact in Python ints
        var = (np.float64(vnum) / (np.float64(N) * np.float64(N))) * (dsc * dsc)
        s = _pow2(float(var + np.float64(np.float32(1e-9))))
        y = acc[m].astype(np.float32) * sc
        xc = y - mean
        o = ((xc * s) * gamma) * np.float32(step)
        out[m] = orc.squareplus_clamp(o.astype(np.float32), -50.0, 50.0)
    return out


@pytest.mark.parametrize("M,N,spread", [(7, 64, 3000), (5, 512, 200000), (6, 1024, 20)])
def test_norm_sqp_oracle_matches_composed_stages(M, N, spread):
    g = np.random.default_rng(N + spread)
    acc = g.integers(-spread, spread + 1, (M, N)).astype(np.int32)
    acc[0] = 0  # zero row: variance 0, the largest scale
    a_scale = (np.logspace(-4, 1, M)).astype(np.float32)
    gamma = (1.0 + 0.1 * g.standard_normal(N)).astype(np.float32)
    out, stats = orc.bitlinear_norm_sqp(acc, a_scale, 2.0 ** -6, gamma, 0.875)
    ref = _composed(acc, a_scale, 2.0 ** -6, gamma, 0.875)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(stats[:, 0], acc.astype(np.int64).sum(1))
    assert np.array_equal(stats[:, 1], (acc.astype(np.int64) ** 2).sum(1))
