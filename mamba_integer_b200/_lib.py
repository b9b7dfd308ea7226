"""ctypes binding of ``libmi_b200.so`` (the C ABI in include/mi_b200.h).

There is no fallback: if the library is missing the import fails with the
command that builds it, and a non-zero status from any entry point raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.path.join(_HERE, "libmi_b200.so")

MI_OK = 0
MI_EPI_I32 = 0
MI_EPI_F32_SCALED = 1
MI_DEV_OVERFLOW = 0x1
MI_DEV_TIMEOUT = 0x2
MI_DEV_PRECOND = 0x4

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float

# name -> argument types (all return int status unless listed in _RESTYPE)
SIGNATURES = {
    "mi_version": [],
    "mi_status_string": [_i],
    "mi_device_error": [ctypes.POINTER(ctypes.c_int), _i, _p],
    "mi_scan_i32": [_p, _p, _p, _p, _i, _p, _p, _p, _i, _i, _i, _i, _p],
    "mi_bitshift_norm": [_p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_quantize_rows": [_p, _i, _i, _i, _p, _i, _p, _p, _p, _p],
    "mi_rowprep": [_p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _i, _i, _p],
    "mi_bitlinear_i8": [_p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p],
    "mi_pack_ternary": [_p, _i, _p, _i, _i, _p],
    "mi_bitlinear_packed": [_p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p],
    "mi_scan_convex_backward": [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_quant_ste_backward": [_p, _p, _p, _i, _i, _p],
    "mi_bitlinear_packed_norm_sqp": [_p, _i, _p, _p, _p, _p, _p, _p, _i, _p, _i, _p, _i, _i, _i, _p],
    "mi_conv_act_quant": [_p, _i, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_conv_act_quant_noalloc": [_p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_conv_act_quant_rows": [_p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_ssm_scan": [_p, _p, _i, _p, _p, _i, _p, _p, _p, _i, _i, _i, _i, _p],
    "mi_ssm_scan_dt": [_p, _p, _i, _p, _i, _p, _p, _p, _i, _p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p],
    "mi_conv_step": [_p, _i, _p, _p, _p, _p, _p, _p, _i, _i, _p],
    "mi_ssm_step": [_p, _p, _i, _i, _p, _p, _p, _i, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_decode_mid": [_p, _i, _p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_decode_mid_packed": [_p, _i, _p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p],
    "mi_argmax_rows": [_p, _i, _i, _i, _p, _p],
    "mi_scan_convex": [_p, _p, _p, _i, _i, _i, _p],
    "mi_squareplus_clamp": [_p, _p, _i64, _f, _f, _p],
    "mi_ste_clamp": [_p, _p, _i64, _f, _f, _p],
    "mi_sigmoid_gate": [_p, _p, _p, _i64, _p],
}
_RESTYPE = {"mi_status_string": ctypes.c_char_p}

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(SO_PATH):
        raise ImportError(f"{SO_PATH} is missing: build it with `python -m mamba_integer_b200.build` "
                          "(nvcc, sm_100a); there is no CPU fallback")
    lib = ctypes.CDLL(SO_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPE.get(name, ctypes.c_int)
    _lib = lib
    return lib


class MIError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != MI_OK:
        msg = load().mi_status_string(rc).decode()
        raise MIError(f"{what} failed: status {rc} ({msg})")


def device_error(stream=None, clear: bool = True) -> int:
    """Device error word (MI_DEV_* bits) of the current device; synchronises."""
    v = ctypes.c_int(0)
    check(load().mi_device_error(ctypes.byref(v), int(clear), stream), "mi_device_error")
    return v.value
