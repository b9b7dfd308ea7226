"""The C-ABI library loads without a GPU and exports every entry point that
include/mi_b200.h declares; the ctypes signature table covers exactly that set.
(include/mi_bpe.h belongs to the tokenizer library, checked in test_tokenizer.py.)"""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "mi_b200.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(mi_\w+)\s*\(", src, flags=re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    from mamba_integer_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"mi_scan_i32", "mi_bitlinear_i8", "mi_rowprep", "mi_ssm_scan", "mi_conv_act_quant"} <= names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_signature_table_matches_header():
    from mamba_integer_b200 import _lib
    assert set(_lib.SIGNATURES) == declared_symbols()


def test_host_side_argument_errors_need_no_gpu(lib):
    # rejected on the host before any CUDA call
    assert lib.mi_scan_i32(None, None, None, None, 15, None, None, None, 1, 1, 16, 16, None) == -1
    assert lib.mi_bitlinear_i8(None, 16, None, None, None, None, None, 16, 16, 16, 16, 0, None) == -1
    assert lib.mi_bitlinear_packed(None, 16, None, None, None, None, None, 16, 16, 16, 64, 0, None) == -1
    assert lib.mi_pack_ternary(None, 16, None, 1, 16, None) == -1
    # the fused scan's kernel variant: 0 (automatic), 1, 2, 3, 4, 8 only (dummy aligned
    # pointers: the call returns before it touches them)
    p = 256
    for split in (5, 6, 7, -1, 16):
        assert lib.mi_ssm_scan_dt(p, p, 32, p, 48, p, p, p, 48, p, 64, p, p, None, None, 1, 8, 64, 16, split,
                                  None) == -1, split
    assert lib.mi_argmax_rows(None, 16, 1, 16, None, None) == -1
    # row conv: at most 4096 channels
    assert lib.mi_conv_act_quant_rows(p, 8200, p, p, p, p, p, 1, 8, 4100, None) == -2
    # the allocation-free conv: one row above its fixed scratch (2^18 rows) is rejected before
    # any CUDA call; xq and xscale are required
    assert lib.mi_conv_act_quant_noalloc(p, 8, p, p, p, p, p, 1, (1 << 18) + 1, 4, None) == -2
    assert lib.mi_conv_act_quant_noalloc(p, 8, p, p, p, p, p, 2, (1 << 17) + 1, 4, None) == -2
    assert lib.mi_conv_act_quant_noalloc(p, 8, p, p, p, None, p, 1, 8, 4, None) == -1
    assert lib.mi_conv_act_quant_noalloc(p, 8, p, p, p, p, None, 1, 8, 4, None) == -1
    # the decode mid kernels: required pointers, d_state 16, D within the cluster
    # layout (a multiple of 64 for the packed weights), dt_rank <= 64, 4-byte aligned
    # packed weights
    def mid_packed(xz=p, w_x=p, R=48, D=2048, N=16, ldx=4096):
        return lib.mi_decode_mid_packed(xz, ldx, p, p, p, w_x, p, R, p, p, p, p, None, p, p, 4, D, N, None)
    assert mid_packed(xz=None) == -1
    assert mid_packed(N=8) == -2
    assert mid_packed(D=2080, ldx=4160) == -2
    assert mid_packed(R=80) == -2
    assert mid_packed(w_x=p + 2) == -1
    assert lib.mi_decode_mid(p, 8200, p, p, p, p, p, 48, p, p, p, p, None, p, p, 4, 4100, 16, None) == -2
    assert lib.mi_version() >= 1
    assert lib.mi_status_string(-2) == b"unsupported shape or configuration"
