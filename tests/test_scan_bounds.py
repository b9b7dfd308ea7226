"""Range facts the fused scan kernel's fast path relies on, checked on the CPU.

ste_clamp(x, lo, hi) = x + (clamp(x) - x) in fp32 (src/mamba_integer_model.py:
136-141) is not clamp(x): for |x| > hi the difference rounds.  The kernel
assumes that ste_clamp(x, -20, 20) never leaves [-36, 36] (the rounding error
is at most half an ulp of x, and once that ulp exceeds 32 the difference
rounds to -x and the result is 0).  Every fp32 value whose exponent can
matter is enumerated here.
"""
import numpy as np


def _ste_clamp(x, lo, hi):
    x = x.astype(np.float32)
    c = np.clip(x, np.float32(lo), np.float32(hi)).astype(np.float32)
    return (x + (c - x).astype(np.float32)).astype(np.float32)


def test_ste_clamp_20_stays_within_36_for_every_fp32_magnitude():
    mant = np.arange(1 << 23, dtype=np.uint32)
    worst = 0.0
    for e in range(127, 127 + 40):  # |x| in [1, 2^40): beyond that the result is 0
        bits = (np.uint32(e) << np.uint32(23)) | mant
        x = bits.view(np.float32)
        for sgn in (1.0, -1.0):
            y = _ste_clamp(np.float32(sgn) * x, -20.0, 20.0)
            assert np.isfinite(y).all()
            worst = max(worst, float(np.abs(y).max()))
    assert worst <= 36.0, worst


def test_ste_clamp_20_is_zero_for_huge_inputs():
    x = np.array([2.0 ** 40, 3.0e38, -2.0 ** 45, -3.0e38], np.float32)
    assert (_ste_clamp(x, -20.0, 20.0) == 0).all()
