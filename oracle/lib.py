"""ctypes wrapper over libmi_oracle.so (test infrastructure only).

Each function takes and returns numpy arrays and calls the C restatement in
``mi_oracle.c``; the docstrings there cite the reference lines each stage
follows.  The library is built by ``make -C oracle`` (also run by
``__graft_entry__.build()``); if it is missing and gcc is present it is built
on first use.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libmi_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def _load():
    global _lib
    if _lib is not None:
        return _lib
    src = os.path.join(_HERE, "mi_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        build()
    lib = ctypes.CDLL(_SO)
    lib.orc_aten_sum.restype = ctypes.c_float
    lib.orc_aten_sum.argtypes = [_f32p, _i64]
    lib.orc_bitshift_norm.restype = None
    lib.orc_bitshift_norm.argtypes = [_f32p, _i64, _i64, _f32p, ctypes.c_float, _f32p, _f32p, ctypes.c_int]
    lib.orc_quant_rows.restype = None
    lib.orc_quant_rows.argtypes = [_f32p, _i64, _i64, _i64, _i8p, _i64, _f32p, ctypes.c_int]
    lib.orc_ternarize.restype = None
    lib.orc_ternarize.argtypes = [_f32p, _i64, ctypes.c_float, _i8p]
    lib.orc_bitlinear.restype = None
    lib.orc_bitlinear.argtypes = [_i8p, _i64, _f32p, _i64, _i64, _i8p, ctypes.c_float, _i64, _f32p, _i64,
                                  _i32p, ctypes.c_int]
    lib.orc_pack_ternary.restype = _i64
    lib.orc_pack_ternary.argtypes = [_i8p, _i64, _i64, _u8p]
    lib.orc_unpack_ternary.restype = None
    lib.orc_unpack_ternary.argtypes = [_u8p, _i64, _i64, _i8p]
    lib.orc_scan_convex_backward.restype = None
    lib.orc_scan_convex_backward.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64,
                                             ctypes.c_int]
    lib.orc_quant_ste_backward.restype = None
    lib.orc_quant_ste_backward.argtypes = [_f32p, _f32p, _f32p, _i64, _i64]
    lib.orc_bitlinear_norm_sqp.restype = None
    lib.orc_bitlinear_norm_sqp.argtypes = [_i32p, _f32p, ctypes.c_float, _f32p, ctypes.c_float, _f32p, _i64p, _i64,
                                           _i64, ctypes.c_int]
    lib.orc_gemm_i8_i32.restype = None
    lib.orc_gemm_i8_i32.argtypes = [_i8p, _i8p, _i32p, _i64, _i64, _i64, ctypes.c_int]
    lib.orc_conv_sqp.restype = None
    lib.orc_conv_sqp.argtypes = [_f32p, _i64, _i64, _i64, _i64, _f32p, _f32p, _f32p, _f32p, ctypes.c_int]
    for name in ("orc_squareplus_clamp", "orc_ste_clamp"):
        fn = getattr(lib, name)
        fn.restype = None
        fn.argtypes = [_f32p, _f32p, _i64, ctypes.c_float, ctypes.c_float]
    lib.orc_sigmoid_gate.restype = None
    lib.orc_sigmoid_gate.argtypes = [_f32p, _f32p, _f32p, _i64]
    lib.orc_scan_convex.restype = None
    lib.orc_scan_convex.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64, ctypes.c_int]
    lib.orc_ssm.restype = None
    lib.orc_ssm.argtypes = [_f32p, _f32p, _i64, _f32p, _f32p, _i64, _f32p, _i64, _i64, _i64, _i64,
                            _f32p, _f32p, ctypes.c_int]
    lib.orc_residual.restype = None
    lib.orc_residual.argtypes = [_f32p, _f32p, ctypes.c_float, _f32p, _i64]
    lib.orc_scale.restype = None
    lib.orc_scale.argtypes = [_f32p, _i64, ctypes.c_float]
    lib.orc_scan_i32.restype = ctypes.c_int
    lib.orc_scan_i32.argtypes = [_i32p, _i32p, _i32p, _i32p, ctypes.c_int, _i64p, _i32p, _i64, _i64, _i64,
                                 _i64, ctypes.c_int]
    _lib = lib
    return lib


def _p(a: np.ndarray, ptype):
    assert a.flags["C_CONTIGUOUS"] or a.ndim == 0, "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ptype)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def aten_sum(row) -> np.float32:
    row = _c(row, np.float32)
    return np.float32(_load().orc_aten_sum(_p(row, _f32p), row.shape[-1]))


def bitshift_norm(x, gamma, step, nthreads=0):
    """BitShiftNorm forward (reference CPU path). x: [..., D] -> (y, inv_rms[rows])."""
    x = _c(x, np.float32)
    D = x.shape[-1]
    T = x.size // D
    y = np.empty_like(x)
    inv = np.empty(T, np.float32)
    _load().orc_bitshift_norm(_p(x, _f32p), T, D, _p(_c(gamma, np.float32), _f32p), float(np.float32(step)),
                              _p(y, _f32p), _p(inv, _f32p), nthreads)
    return y, inv


def quant_rows(x, nthreads=0):
    """activation_quant_dynamic: x [..., K] -> (xq int8 [..., K], x_scale fp32 [rows])."""
    x = _c(x, np.float32)
    K = x.shape[-1]
    T = x.size // K
    xq = np.empty(x.shape, np.int8)
    xs = np.empty(T, np.float32)
    _load().orc_quant_rows(_p(x, _f32p), K, T, K, _p(xq, _i8p), K, _p(xs, _f32p), nthreads)
    return xq, xs


def ternarize(w, scale):
    w = _c(w, np.float32)
    q = np.empty(w.shape, np.int8)
    _load().orc_ternarize(_p(w, _f32p), w.size, float(np.float32(scale)), _p(q, _i8p))
    return q


def bitlinear(xq, xscale, wq, w_scale, want_acc=False, nthreads=0):
    """F.linear(xq, wq) * (w_scale * x_scale): xq [T,K] int8, wq [N,K] int8 -> fp32 [T,N]."""
    xq = _c(xq, np.int8)
    K = xq.shape[-1]
    T = xq.size // K
    wq = _c(wq, np.int8)
    N = wq.shape[0]
    out = np.empty((T, N), np.float32)
    acc = np.empty((T, N), np.int32) if want_acc else None
    _load().orc_bitlinear(_p(xq, _i8p), K, _p(_c(xscale, np.float32), _f32p), T, K, _p(wq, _i8p),
                          float(np.float32(w_scale)), N, _p(out, _f32p), N,
                          _p(acc, _i32p) if want_acc else None, nthreads)
    return (out, acc) if want_acc else out


def pack_ternary(W):
    """int8 ternary [N, K] -> 2-bit packed [N, K/4] uint8 and the count of
    values outside {-1, 0, 1}."""
    W = _c(W, np.int8)
    N, K = W.shape
    assert K % 16 == 0
    Wp = np.empty((N, K // 4), np.uint8)
    bad = _load().orc_pack_ternary(_p(W, _i8p), N, K, _p(Wp, _u8p))
    return Wp, int(bad)


def unpack_ternary(Wp, K):
    Wp = _c(Wp, np.uint8)
    N = Wp.shape[0]
    W = np.empty((N, K), np.int8)
    _load().orc_unpack_ternary(_p(Wp, _u8p), N, K, _p(W, _i8p))
    return W


def gemm_i8_i32(A, W, nthreads=0):
    A = _c(A, np.int8)
    W = _c(W, np.int8)
    M, K = A.shape
    N = W.shape[0]
    C = np.empty((M, N), np.int32)
    _load().orc_gemm_i8_i32(_p(A, _i8p), _p(W, _i8p), _p(C, _i32p), M, N, K, nthreads)
    return C


def scan_convex_backward(grad_h, h, u, nums, nthreads=0):
    """Training-side convex scan backward: (grad_u, grad_nums), each [B, L, DN] fp32."""
    grad_h, h, u, nums = (_c(a, np.float32) for a in (grad_h, h, u, nums))
    Bsz, L, DN = grad_h.shape
    gu = np.empty_like(grad_h)
    gn = np.empty_like(grad_h)
    _load().orc_scan_convex_backward(_p(grad_h, _f32p), _p(h, _f32p), _p(u, _f32p), _p(nums, _f32p), _p(gu, _f32p),
                                     _p(gn, _f32p), Bsz, L, DN, nthreads)
    return gu, gn


def quant_ste_backward(grad_xq, amax):
    """Training-side STE backward of the activation quantisation: grad_x [T, K]."""
    grad_xq = _c(grad_xq, np.float32)
    amax = _c(amax, np.float32)
    T, K = grad_xq.shape
    gx = np.empty_like(grad_xq)
    _load().orc_quant_ste_backward(_p(grad_xq, _f32p), _p(amax, _f32p), _p(gx, _f32p), T, K)
    return gx


def bitlinear_norm_sqp(acc, a_scale, w_scale, gamma, step, nthreads=0):
    """Config-3 epilogue on int32 accumulators [M, N]: (out fp32 [M, N], stats int64 [M, 2])."""
    acc = _c(acc, np.int32)
    M, N = acc.shape
    a_scale = _c(a_scale, np.float32)
    gamma = _c(gamma, np.float32)
    out = np.empty((M, N), np.float32)
    stats = np.empty((M, 2), np.int64)
    _load().orc_bitlinear_norm_sqp(_p(acc, _i32p), _p(a_scale, _f32p), float(np.float32(w_scale)),
                                   _p(gamma, _f32p), float(np.float32(step)), _p(out, _f32p), _p(stats, _i64p), M,
                                   N, nthreads)
    return out, stats


def conv_sqp(x, w, bias, nthreads=0):
    """Causal depthwise conv (bias, then FMA taps) + ste_clamp(+-50) + squareplus.

    x: [Bsz, L, D] -> (conv_out, act_out) each [Bsz, L, D]."""
    x = _c(x, np.float32)
    Bsz, L, D = x.shape
    co = np.empty_like(x)
    ao = np.empty_like(x)
    _load().orc_conv_sqp(_p(x, _f32p), D, Bsz, L, D, _p(_c(w, np.float32).reshape(D, 4), _f32p),
                         _p(_c(bias, np.float32), _f32p), _p(co, _f32p), _p(ao, _f32p), nthreads)
    return co, ao


def squareplus_clamp(x, lo=-50.0, hi=50.0):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    _load().orc_squareplus_clamp(_p(x, _f32p), _p(y, _f32p), x.size, lo, hi)
    return y


def ste_clamp(x, lo, hi):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    _load().orc_ste_clamp(_p(x, _f32p), _p(y, _f32p), x.size, lo, hi)
    return y


def sigmoid_gate(y, z):
    y = _c(y, np.float32)
    z = _c(z, np.float32)
    o = np.empty_like(y)
    _load().orc_sigmoid_gate(_p(y, _f32p), _p(z, _f32p), _p(o, _f32p), y.size)
    return o


def scan_convex(u, nums, nthreads=0):
    """DyadicScanFunction CPU forward: u, nums [B, L, DN] -> h [B, L, DN]."""
    u = _c(u, np.float32)
    nums = _c(nums, np.float32)
    Bsz, L, DN = u.shape
    h = np.empty_like(u)
    _load().orc_scan_convex(_p(u, _f32p), _p(nums, _f32p), _p(h, _f32p), Bsz, L, DN, nthreads)
    return h


def ssm(xact, bc, modraw, z, base, Bsz, L, want_h=False, nthreads=0):
    """Fused SSM section: xact [T,D], bc [T,2N] (B|C), modraw [T,D], z [T,D], base [D,N]."""
    xact = _c(xact, np.float32)
    bc = _c(bc, np.float32)
    modraw = _c(modraw, np.float32)
    z = _c(z, np.float32)
    base = _c(base, np.float32)
    D, N = base.shape
    out = np.empty((Bsz * L, D), np.float32)
    hl = np.empty((Bsz, D, N), np.float32) if want_h else None
    _load().orc_ssm(_p(xact, _f32p), _p(bc, _f32p), bc.shape[-1], _p(modraw, _f32p), _p(z, _f32p),
                    z.shape[-1], _p(base, _f32p), Bsz, L, D, N, _p(out, _f32p),
                    _p(hl, _f32p) if want_h else None, nthreads)
    return (out, hl) if want_h else out


def residual(res, out, g):
    res = _c(res, np.float32)
    out = _c(out, np.float32)
    y = np.empty_like(res)
    _load().orc_residual(_p(res, _f32p), _p(out, _f32p), float(np.float32(g)), _p(y, _f32p), res.size)
    return y


def scale_(x, s):
    assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"]
    _load().orc_scale(_p(x, _f32p), x.size, float(np.float32(s)))
    return x


def scan_i32(x, B, C, n, k=15, h0=None, nthreads=0):
    """Integer dyadic scan: x [Bsz,L,D], B/C [Bsz,L,N], n [D,N] int32 -> (y int64 [Bsz,L,D], h_T int32)."""
    x = _c(x, np.int32)
    B = _c(B, np.int32)
    C = _c(C, np.int32)
    n = _c(n, np.int32)
    Bsz, L, D = x.shape
    N = n.shape[1]
    h = np.zeros((Bsz, D, N), np.int32) if h0 is None else _c(h0, np.int32).copy()
    y = np.empty((Bsz, L, D), np.int64)
    rc = _load().orc_scan_i32(_p(x, _i32p), _p(B, _i32p), _p(C, _i32p), _p(n, _i32p), int(k), _p(y, _i64p),
                              _p(h, _i32p), Bsz, L, D, N, nthreads)
    if rc != 0:
        raise OverflowError(f"orc_scan_i32 failed with status {rc}")
    return y, h
