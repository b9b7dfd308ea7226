"""The bounded squareplus of the conv, the scan's decay prologue and the
decode step skips the upper clamp (r <= 1e3) of each Newton step of the
reference's reciprocal square root (src/mamba_integer_model.py:80-102, the
rational squareplus at :105-121).  For y = x*x + 4 >= 4 and a first guess
<= 0.5, each step multiplies r by at most fl(1.5), so r never comes near 1e3;
a NaN or infinite y gives the same r either way.  Checked here in fp32 (every
operation rounded, as the kernels round it) over every exponent of |x| < 256
with a stride of mantissas, the guess thresholds, and special values."""
import numpy as np

F = np.float32


def _clampf(v, lo, hi):
    """torch.clamp on fp32: NaN stays NaN."""
    return np.where(np.isnan(v), v, np.minimum(np.maximum(v, F(lo)), F(hi))).astype(F)


def _squareplus(x, upper_clamp):
    with np.errstate(all="ignore"):
        y = (x * x).astype(F) + F(4)
        y = y.astype(F)
        r = np.where(y > F(16), F(0.125), F(0.5)).astype(F)
        r = np.where(y > F(64), F(0.0625), r).astype(F)
        r = np.where(y > F(256), F(0.03125), r).astype(F)
        for _ in range(3):
            t = (F(0.5) * y).astype(F)
            t = (t * r).astype(F)
            t = (t * r).astype(F)
            t = (F(1.5) - t).astype(F)
            r = (r * t).astype(F)
            r = _clampf(r, 1e-6, 1e3) if upper_clamp else _clampf(r, 1e-6, np.inf)
        s = _clampf((y * r).astype(F), 0.0, 1e3)
        return (F(0.5) * (x + s).astype(F)).astype(F)


def _same_bits(a, b):
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_upper_newton_clamp_never_binds():
    mant = np.arange(0, 1 << 23, 61, dtype=np.uint32)  # a stride of mantissas per exponent
    for e in range(0, 127 + 8):  # |x| from the subnormals up to 2^8
        bits = (np.uint32(e) << np.uint32(23)) | mant
        x = bits.view(F)
        for sgn in (F(1), F(-1)):
            v = (sgn * x).astype(F)
            assert _same_bits(_squareplus(v, True), _squareplus(v, False)), e


def test_upper_newton_clamp_special_values():
    special = [0.0, -0.0, np.inf, -np.inf, np.nan, 3.4e38, -3.4e38, 1e19, 2e19, 1e-45]
    # +-64 ulps around the x where x*x + 4 crosses the guess thresholds 16, 64, 256
    near = [(np.array([np.sqrt(F(c))], dtype=F).view(np.uint32) + np.arange(-64, 65, dtype=np.int64)
             ).astype(np.uint32).view(F) for c in (12.0, 60.0, 252.0)]
    v = np.concatenate([np.array(special, dtype=F)] + near).astype(F)
    v = np.concatenate([v, -v])
    a, b = _squareplus(v, True), _squareplus(v, False)
    assert np.array_equal(np.isnan(a), np.isnan(b))
    assert _same_bits(a[~np.isnan(a)], b[~np.isnan(b)])
