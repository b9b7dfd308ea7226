"""The 2-bit packed ternary weight format, on the CPU (oracle side).

Known-answer vectors written out by hand from the format's definition: the
little-endian 32-bit word g of a row holds weights 16g .. 16g+15, weight
16g + 4q + j in bits [p, p + 2) with p = 4j + 2(q & 1) + 16(q >> 1),
00 = 0, 01 = +1, 11 = -1.
"""
import numpy as np

from oracle import lib as orc


def test_pack_known_answer():
    w = np.zeros((1, 32), np.int8)
    w[0, 0] = 1     # q=0 j=0 -> bits 0-1   = 01
    w[0, 1] = -1    # q=0 j=1 -> bits 4-5   = 11
    w[0, 4] = 1     # q=1 j=0 -> bits 2-3   = 01
    w[0, 15] = -1   # q=3 j=3 -> bits 30-31 = 11
    w[0, 16 + 10] = 1  # second word: q=2 j=2 -> bits 24-25 = 01
    wp, bad = orc.pack_ternary(w)
    assert bad == 0
    assert wp.tolist() == [[0x35, 0x00, 0x00, 0xC0, 0x00, 0x00, 0x00, 0x01]]


def test_pack_unpack_round_trip_and_bad_values():
    rng = np.random.default_rng(7)
    w = rng.integers(-1, 2, size=(37, 192)).astype(np.int8)
    wp, bad = orc.pack_ternary(w)
    assert bad == 0 and wp.shape == (37, 48)
    assert np.array_equal(orc.unpack_ternary(wp, 192), w)
    w[3, 5] = 2
    w[9, 100] = -128
    wp2, bad2 = orc.pack_ternary(w)
    assert bad2 == 2
    back = orc.unpack_ternary(wp2, 192)
    assert back[3, 5] == 0 and back[9, 100] == 0


def test_packed_gemm_equals_dense_gemm_on_cpu():
    rng = np.random.default_rng(3)
    a = rng.integers(-127, 128, size=(9, 128)).astype(np.int8)
    w = rng.integers(-1, 2, size=(16, 128)).astype(np.int8)
    wp, _ = orc.pack_ternary(w)
    assert np.array_equal(orc.gemm_i8_i32(a, orc.unpack_ternary(wp, 128)), orc.gemm_i8_i32(a, w))
