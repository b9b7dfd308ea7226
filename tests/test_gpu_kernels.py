"""GPU kernels against the CPU oracle, stage by stage, through the C ABI.
Integer outputs must be identical; float stages too (the kernels replay the
reference's floating-point order, so the tolerance is zero ulp)."""
import numpy as np
import pytest
import torch

import cases
from oracle import lib as orc

pytestmark = pytest.mark.gpu


def _mi():
    from mamba_integer_b200 import _lib, kernels
    _lib.load()
    return kernels


def _eq(a, b, what=""):
    a = a.detach().cpu().numpy() if torch.is_tensor(a) else a
    b = b.detach().cpu().numpy() if torch.is_tensor(b) else b
    assert a.shape == b.shape, (what, a.shape, b.shape)
    bad = a.view(np.uint8) != b.view(np.uint8) if a.dtype == b.dtype else a != b
    if bad.any():
        idx = np.argwhere(a != b)[:5]
        raise AssertionError(f"{what}: {int((a != b).sum())} mismatches, first at {idx.tolist()}")


# ---------------------------------------------------------------- integer scan
@pytest.mark.parametrize("bsz,L,D", [(2, 300, 200), (1, 33, 64), (3, 1, 4), (2, 4096, 128), (4, 37, 2400)])
def test_scan_i32_matches_oracle(cuda_dev, bsz, L, D):
    k = _mi()
    g = torch.Generator().manual_seed(bsz * 1000 + L + D)
    q = lambda *s: torch.round(torch.randn(*s, generator=g) * 32).clamp(-127, 127).to(torch.int32)  # noqa: E731
    x, B, C = q(bsz, L, D), q(bsz, L, 16), q(bsz, L, 16)
    n = torch.randint(29492, 32736, (D, 16), generator=g, dtype=torch.int32)
    n[0, 0], n[0, 1] = 0, 32768  # decay 0 and decay 1 edges
    h0 = torch.randint(-2 ** 20, 2 ** 20, (bsz, D, 16), generator=g, dtype=torch.int32)
    y_ref, h_ref = orc.scan_i32(x.numpy(), B.numpy(), C.numpy(), n.numpy(), 15, h0=h0.numpy())
    dv = [t.to(cuda_dev) for t in (x, B, C, n, h0)]
    y64, h64 = k.scan_i32(*dv[:4], 15, h0=dv[4], y_dtype=torch.int64)
    _eq(y64, y_ref, "y64")
    _eq(h64, h_ref, "h")
    if np.abs(y_ref).max() < 2 ** 31:
        y32, h32 = k.scan_i32(*dv[:4], 15, h0=dv[4], y_dtype=torch.int32)
        _eq(y32, y_ref.astype(np.int32), "y32")
        _eq(h32, h_ref, "h32")


@pytest.mark.parametrize("bsz,D", [(4, 2400), (1, 64)])  # 2 and 4 lanes per channel
def test_scan_i32_full_input_range(cuda_dev, bsz, D):
    """B and C over the whole stated range +-32767 (the kernel repacks them as 16-bit pairs)."""
    k = _mi()
    L = 50
    g = torch.Generator().manual_seed(D + bsz)
    B = torch.randint(-32767, 32768, (bsz, L, 16), generator=g, dtype=torch.int32)
    C = torch.randint(-32767, 32768, (bsz, L, 16), generator=g, dtype=torch.int32)
    B[0, 0, :2], C[0, 0, :2] = torch.tensor([32767, -32767]), torch.tensor([-32767, 32767])
    x = torch.randint(-3, 4, (bsz, L, D), generator=g, dtype=torch.int32)
    n = torch.randint(0, 32769, (D, 16), generator=g, dtype=torch.int32)
    y_ref, h_ref = orc.scan_i32(x.numpy(), B.numpy(), C.numpy(), n.numpy(), 15)
    y64, h64 = k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), 15, y_dtype=torch.int64)
    _eq(y64, y_ref, "y64")
    _eq(h64, h_ref, "h")


def test_scan_i32_config2_distribution(cuda_dev):
    """Config 2's input distribution at a reduced size from zero states: every
    chunk takes the 32-bit path, and every warp but channel 0's has all decays
    >= 2^(k-1) (the folded add-back)."""
    k = _mi()
    bsz, L, D = 2, 512, 256
    g = torch.Generator().manual_seed(5)
    q = lambda *s: torch.round(torch.randn(*s, generator=g) * 32).clamp(-127, 127).to(torch.int32)  # noqa: E731
    x, B, C = q(bsz, L, D), q(bsz, L, 16), q(bsz, L, 16)
    n = torch.randint(int(0.90 * 2 ** 15), int(0.999 * 2 ** 15) + 1, (D, 16), generator=g, dtype=torch.int32)
    n[0, 5] = 2 ** 14 - 1
    y_ref, h_ref = orc.scan_i32(x.numpy(), B.numpy(), C.numpy(), n.numpy(), 15)
    y, h = k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), 15, y_dtype=torch.int32)
    _eq(y, y_ref.astype(np.int32), "y32")
    _eq(h, h_ref, "h")


@pytest.mark.parametrize("kk", [1, 7, 15, 30])
def test_scan_i32_shift_amounts(cuda_dev, kk):
    """Every k the API takes, with n at 0, 2^(k-1)-1, 2^(k-1) and 2^k (where the
    kernel's multiply-high form of (h*n) >> k changes case) and large states."""
    k = _mi()
    bsz, L, D = 2, 100, 64
    g = torch.Generator().manual_seed(kk)
    q = lambda *s: torch.round(torch.randn(*s, generator=g) * 32).clamp(-127, 127).to(torch.int32)  # noqa: E731
    x, B, C = q(bsz, L, D), q(bsz, L, 16), q(bsz, L, 16)
    n = torch.randint(0, 2 ** kk + 1, (D, 16), generator=g, dtype=torch.int32)
    n[0, :4] = torch.tensor([0, max(2 ** (kk - 1) - 1, 0), 2 ** (kk - 1), 2 ** kk])
    h0 = torch.randint(-2 ** 28, 2 ** 28, (bsz, D, 16), generator=g, dtype=torch.int32)
    y_ref, h_ref = orc.scan_i32(x.numpy(), B.numpy(), C.numpy(), n.numpy(), kk, h0=h0.numpy())
    y64, h64 = k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), kk, h0=h0.to(cuda_dev), y_dtype=torch.int64)
    _eq(y64, y_ref, "y64")
    _eq(h64, h_ref, "h")


@pytest.mark.parametrize("y_dtype", [torch.int64, torch.int32])
def test_scan_i32_chunk_paths_switch(cuda_dev, y_dtype):
    """Large initial states (chunks whose bound does not rule out an int32
    overflow: 64-bit y sums, checked adds) that decay within a few chunks to
    states where the 32-bit path applies; one sequence crosses over."""
    k = _mi()
    bsz, L, D = 3, 400, 96
    g = torch.Generator().manual_seed(77)
    q = lambda *s: torch.round(torch.randn(*s, generator=g) * 32).clamp(-127, 127).to(torch.int32)  # noqa: E731
    x, B, C = q(bsz, L, D), q(bsz, L, 16), q(bsz, L, 16)
    n = torch.randint(0, 2 ** 14 + 1, (D, 16), generator=g, dtype=torch.int32)  # decay <= 1/2
    hbits = 30 if y_dtype == torch.int64 else 21  # int32 y: 16 * 127 * 2^21 > 2^31 still needs the wide path
    h0 = torch.randint(-2 ** hbits, 2 ** hbits, (bsz, D, 16), generator=g, dtype=torch.int32)
    h0[1] = 0  # this sequence starts small
    y_ref, h_ref = orc.scan_i32(x.numpy(), B.numpy(), C.numpy(), n.numpy(), 15, h0=h0.numpy())
    if y_dtype == torch.int32:
        assert np.abs(y_ref).max() < 2 ** 31
        y_ref = y_ref.astype(np.int32)
    y, h = k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), 15, h0=h0.to(cuda_dev), y_dtype=y_dtype)
    _eq(y, y_ref, "y")
    _eq(h, h_ref, "h")


def test_scan_i32_kat_negative_floor(cuda_dev):
    """h = -1, n = 1, k = 15: (-1*1) >> 15 = -1 (floor), not 0 (truncation)."""
    k = _mi()
    x = torch.zeros(1, 3, 4, dtype=torch.int32)
    B = torch.zeros(1, 3, 16, dtype=torch.int32)
    C = torch.zeros(1, 3, 16, dtype=torch.int32)
    C[..., 0] = 1
    n = torch.ones(4, 16, dtype=torch.int32)
    h0 = torch.full((1, 4, 16), -1, dtype=torch.int32)
    y, h = k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), 15, h0=h0.to(cuda_dev), y_dtype=torch.int64)
    assert (h.cpu() == -1).all() and (y.cpu() == -1).all()


def test_scan_i32_overflow_is_reported(cuda_dev):
    k = _mi()
    x = torch.full((1, 2, 4), 127, dtype=torch.int32)
    B = torch.full((1, 2, 16), 127, dtype=torch.int32)
    C = torch.ones(1, 2, 16, dtype=torch.int32)
    n = torch.full((4, 16), 32768, dtype=torch.int32)
    h0 = torch.full((1, 4, 16), 2 ** 31 - 100, dtype=torch.int32)
    with pytest.raises(OverflowError):
        k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), 15, h0=h0.to(cuda_dev), y_dtype=torch.int64)
    x[0, 0, 0] = 40000  # outside the stated input range
    with pytest.raises(OverflowError):
        k.scan_i32(*(t.to(cuda_dev) for t in (x, B, C, n)), 15, y_dtype=torch.int64)


# ---------------------------------------------------------------- row stages
@pytest.mark.parametrize("D", [256, 768, 1024, 32, 96])
def test_bitshift_norm_matches_oracle(cuda_dev, D):
    k = _mi()
    g = torch.Generator().manual_seed(D)
    x = torch.randn(333, D, generator=g) * torch.logspace(-3, 2.5, 333).unsqueeze(1) + torch.randn(333, 1, generator=g)
    gamma = 1 + 0.1 * torch.randn(D, generator=g)
    step = torch.tensor([0.875])
    y_ref, inv_ref = orc.bitshift_norm(x.numpy(), gamma.numpy(), 0.875)
    y, inv = k.bitshift_norm(x.to(cuda_dev), gamma.to(cuda_dev), step.to(cuda_dev))
    _eq(y, y_ref, "norm y")
    _eq(inv, inv_ref, "inv_rms")


def test_norm_fixture_inputs(cuda_dev):
    k = _mi()
    x, g, st = cases.norm_inputs()
    gold = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "stages.npz"))
    y, inv = k.bitshift_norm(torch.from_numpy(x).to(cuda_dev), torch.from_numpy(g).to(cuda_dev),
                             torch.from_numpy(st).to(cuda_dev))
    _eq(y, gold["norm.y"], "norm y vs reference fixture")
    _eq(inv, gold["norm.inv_rms"], "inv_rms vs reference fixture")


@pytest.mark.parametrize("K", [256, 48, 1536, 80])
def test_quantize_rows_matches_oracle(cuda_dev, K):
    k = _mi()
    x = cases.quant_inputs()[:, :K] if K <= 256 else np.random.default_rng(K).standard_normal((77, K)).astype(np.float32)
    x = np.ascontiguousarray(x)
    q_ref, s_ref = orc.quant_rows(x)
    q, s = k.quantize_rows(torch.from_numpy(x).to(cuda_dev))
    _eq(q, q_ref, "xq")
    _eq(s, s_ref, "xscale")


@pytest.mark.parametrize("K", [1, 7, 33, 64])
def test_quantize_rows_narrow_strided(cuda_dev, K):
    """Rows of at most 64 values (two per warp) read from a wider strided
    array: ragged widths, a NaN row, zero and infinite rows, row counts that
    leave a warp half empty."""
    k = _mi()
    g = np.random.default_rng(K)
    T = 301
    wide = (g.standard_normal((T, K + 5)) * np.logspace(-3, 3, T)[:, None]).astype(np.float32)
    wide[3, :K] = 0.0
    wide[4, K // 2] = np.nan
    wide[5, 0] = np.inf
    wide[6, :K] = 127.0 / 3
    x = np.ascontiguousarray(wide[:, :K])
    q_ref, s_ref = orc.quant_rows(x)
    xd = torch.from_numpy(wide).to(cuda_dev)[:, :K]
    q, s = k.quantize_rows(xd)
    _eq(q, q_ref, "xq")
    # the NaN row's scale is NaN on both sides; its payload bits are not specified
    s = s.cpu().numpy()
    assert np.array_equal(np.isnan(s), np.isnan(s_ref))
    _eq(s[~np.isnan(s)], s_ref[~np.isnan(s_ref)], "xscale")


@pytest.mark.parametrize("K", [48, 200])
def test_quantize_rows_clears_the_given_rows(cuda_dev, K):
    # the dt quantisation zero-fills the fused scan's row-maximum array on the way,
    # without changing its own outputs (narrow and wide rows)
    k = _mi()
    g = np.random.default_rng(3 + K)
    x = g.standard_normal((257, K)).astype(np.float32)
    q_ref, s_ref = orc.quant_rows(x)
    xd = torch.from_numpy(x).to(cuda_dev)
    clear = torch.full((257,), 5.0, device=cuda_dev)
    q, s = k.quantize_rows(xd, clear=clear)
    _eq(q, q_ref, "xq")
    _eq(s, s_ref, "xscale")
    assert torch.equal(clear, torch.zeros_like(clear))


@pytest.mark.parametrize("D", [256, 768])
def test_rowprep_fused_matches_oracle(cuda_dev, D):
    k = _mi()
    g = torch.Generator().manual_seed(7 + D)
    T = 515
    res = torch.randn(T, D, generator=g) * 3
    out = torch.randn(T, D, generator=g)
    gate = torch.tensor([0.144337567])
    gamma = 1 + 0.05 * torch.randn(D, generator=g)
    step = torch.tensor([1.0625])
    newres = orc.residual(res.numpy(), out.numpy(), gate.numpy()[0])
    y_ref, _ = orc.bitshift_norm(newres, gamma.numpy(), 1.0625)
    q_ref, s_ref = orc.quant_rows(y_ref)
    dv = lambda t: t.to(cuda_dev).contiguous()  # noqa: E731
    xo = torch.empty(T, D, device=cuda_dev)
    yn = torch.empty(T, D, device=cuda_dev)
    xq = torch.empty(T, D, dtype=torch.int8, device=cuda_dev)
    xs = torch.empty(T, device=cuda_dev)
    k.rowprep(dv(gamma), dv(step), T, D, x=dv(res), delta=dv(out), res_gate=dv(gate), x_out=xo, y_norm=yn, xq=xq,
              xscale=xs)
    _eq(xo, newres, "residual")
    _eq(yn, y_ref, "norm")
    _eq(xq, q_ref, "xq")
    _eq(xs, s_ref, "xscale")
    # embedding-gather variant
    emb = torch.randn(1000, D, generator=g)
    ids = torch.randint(0, 1000, (T,), generator=g)
    y2, _ = orc.bitshift_norm(emb.numpy()[ids.numpy()], gamma.numpy(), 1.0625)
    q2, s2 = orc.quant_rows(y2)
    k.rowprep(dv(gamma), dv(step), T, D, ids=dv(ids), emb=dv(emb), x_out=xo, xq=xq, xscale=xs)
    _eq(xo, emb.numpy()[ids.numpy()], "gather")
    _eq(xq, q2, "xq gather")
    _eq(xs, s2, "xscale gather")


# ---------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (300, 3072, 768), (1000, 80, 1536), (257, 1536, 48),
                                   (640, 768, 1536), (129, 4096, 256), (512, 96, 64)])
def test_gemm_i8_matches_oracle(cuda_dev, M, N, K):
    k = _mi()
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    W = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    ref = orc.gemm_i8_i32(A.numpy(), W.numpy())
    acc = k.bitlinear_i8(A.to(cuda_dev), W.to(cuda_dev))
    _eq(acc, ref, "int32 accumulators")
    xs = (torch.rand(M, generator=g) * 0.05 + 1e-3)
    ws = torch.tensor([2.0 ** -6])
    out_ref = orc.bitlinear(A.numpy(), xs.numpy(), W.numpy(), 2.0 ** -6)
    out = k.bitlinear_i8(A.to(cuda_dev), W.to(cuda_dev), xs.to(cuda_dev), ws.to(cuda_dev))
    _eq(out, out_ref, "scaled fp32")
    os_ = torch.tensor([np.float32(1 / np.sqrt(768))])
    out2 = k.bitlinear_i8(A.to(cuda_dev), W.to(cuda_dev), xs.to(cuda_dev), ws.to(cuda_dev), out_scale=os_.to(cuda_dev))
    _eq(out2, (out_ref * os_.numpy()[0]).astype(np.float32), "output scale")


def test_gemm_config3_slice(cuda_dev):
    """BitLinear config 3 inputs (activation quant of N(0,1), ternary W): a 1024-row slice."""
    from mamba_integer_b200 import synth
    k = _mi()
    A, a_scale, Wq, ws = synth.bitlinear_inputs(M=1024, K=2048, N=1024)
    ref = orc.gemm_i8_i32(A.numpy(), Wq.numpy())
    _eq(k.bitlinear_i8(A.to(cuda_dev), Wq.to(cuda_dev)), ref, "config-3 slice")


# ---------------------------------------------------------------- 2-bit packed weights
@pytest.mark.parametrize("N,K", [(80, 1536), (3, 16), (257, 48), (1024, 2048)])
def test_pack_ternary_matches_oracle(cuda_dev, N, K):
    from mamba_integer_b200 import _lib
    k = _mi()
    g = torch.Generator().manual_seed(N + K)
    W = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    ref, bad = orc.pack_ternary(W.numpy())
    assert bad == 0
    _eq(k.pack_ternary(W.to(cuda_dev)), ref, "packed bytes")
    assert _lib.device_error() == 0


def test_pack_ternary_flags_non_ternary_values(cuda_dev):
    from mamba_integer_b200 import _lib
    k = _mi()
    W = torch.zeros(2, 32, dtype=torch.int8)
    W[0, 3], W[1, 17], W[1, 0] = 2, -5, -1
    ref, bad = orc.pack_ternary(W.numpy())
    assert bad == 2
    _lib.device_error()  # clear
    _eq(k.pack_ternary(W.to(cuda_dev)), ref, "packed bytes with invalid values stored as 0")
    assert _lib.device_error() & _lib.MI_DEV_PRECOND


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (300, 3072, 768), (1000, 80, 1536), (640, 768, 1536),
                                   (129, 4096, 256), (512, 96, 64), (200, 32, 192), (130, 256, 2048)])
def test_gemm_packed_matches_oracle(cuda_dev, M, N, K):
    k = _mi()
    g = torch.Generator().manual_seed(M * 5 + N * 11 + K)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    W = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    Wp = torch.from_numpy(orc.pack_ternary(W.numpy())[0])
    ref = orc.gemm_i8_i32(A.numpy(), W.numpy())
    _eq(k.bitlinear_packed(A.to(cuda_dev), Wp.to(cuda_dev)), ref, "int32 accumulators (packed weights)")
    xs = (torch.rand(M, generator=g) * 0.05 + 1e-3)
    ws = torch.tensor([2.0 ** -6])
    out_ref = orc.bitlinear(A.numpy(), xs.numpy(), W.numpy(), 2.0 ** -6)
    out = k.bitlinear_packed(A.to(cuda_dev), Wp.to(cuda_dev), xs.to(cuda_dev), ws.to(cuda_dev))
    _eq(out, out_ref, "scaled fp32 (packed weights)")


@pytest.mark.parametrize("M,N,K", [(4736, 1024, 832), (2176, 1152, 832), (4736, 1024, 768), (300, 1152, 768)])
def test_gemm_wide_tiles_both_weight_formats(cuda_dev, M, N, K):
    """Kernel choices by shape: 256-wide tiles (N % 256 == 0 and enough
    tiles), 128-wide tiles, and the A-resident kernel (K <= 768, N > 128, no
    256-wide tiling)."""
    k = _mi()
    g = torch.Generator().manual_seed(M + N)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    W = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    xs = (torch.rand(M, generator=g) * 0.05 + 1e-3)
    ws = torch.tensor([2.0 ** -6])
    out_ref = orc.bitlinear(A.numpy(), xs.numpy(), W.numpy(), 2.0 ** -6)
    Ad, Wd, xsd, wsd = A.to(cuda_dev), W.to(cuda_dev), xs.to(cuda_dev), ws.to(cuda_dev)
    _eq(k.bitlinear_i8(Ad, Wd, xsd, wsd), out_ref, "int8 weights")
    _eq(k.bitlinear_packed(Ad, k.pack_ternary(Wd), xsd, wsd), out_ref, "packed weights")


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 512), (4000, 4096, 320), (16384, 768, 1536), (1100, 32768, 768)])
def test_gemm_pair_kernel_matches_oracle(cuda_dev, M, N, K, monkeypatch):
    """The 2-SM kernel (tcgen05.mma.cta_group::2, 256 x 256 tiles over an SM pair), chosen
    for int8 weights and N % 256 == 0 with a tile per pair: int32, scaled and
    out_scale outputs, ragged M (a pair whose second half is past M), a K tail; the
    one-CTA kernels (MI_GEMM_2SM=0, and packed weights always) give the same bits."""
    k = _mi()
    g = torch.Generator().manual_seed(M + N + K)
    A = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    W = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    xs = (torch.rand(M, generator=g) * 0.05 + 1e-3)
    acc_ref = orc.gemm_i8_i32(A.numpy(), W.numpy())
    out_ref = orc.bitlinear(A.numpy(), xs.numpy(), W.numpy(), 2.0 ** -6)
    Ad, Wd, xsd = A.to(cuda_dev), W.to(cuda_dev), xs.to(cuda_dev)
    wsd, osd = torch.tensor([2.0 ** -6], device=cuda_dev), torch.tensor([0.125], device=cuda_dev)
    Wp = k.pack_ternary(Wd)
    for pair in ("1", "0"):
        monkeypatch.setenv("MI_GEMM_2SM", pair)
        _eq(k.bitlinear_i8(Ad, Wd), acc_ref, f"int8 weights, int32 out, pair={pair}")
        _eq(k.bitlinear_packed(Ad, Wp), acc_ref, f"packed weights, int32 out, pair={pair}")
        _eq(k.bitlinear_packed(Ad, Wp, xsd, wsd), out_ref, f"packed weights, scaled out, pair={pair}")
        scaled = k.bitlinear_i8(Ad, Wd, xsd, wsd, out_scale=osd).cpu().numpy()
        _eq(scaled, (out_ref * np.float32(0.125)).astype(np.float32), f"int8 weights, out_scale, pair={pair}")
    from mamba_integer_b200 import _lib
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(16384, 768, 1536), (4096, 768, 1536), (16384, 3072, 768)])
def test_ternary_matmul_weight_form_rule(cuda_dev, M, N, K):
    """ternary_matmul takes the int8 copy on the 2-SM kernel for a compute-heavy GEMM
    (the config-4 out_proj shape, K 1536, at prefill size) and the packed weights
    otherwise (fewer rows; K 768): either way the bits of the packed kernel."""
    from mamba_integer_b200.rational_bitnet import TernaryWeights, _pair_kernel_wins, ternary_matmul
    k = _mi()
    g = torch.Generator().manual_seed(M + N + K)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(cuda_dev)
    W = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8).to(cuda_dev)
    xs = (torch.rand(M, generator=g) * 0.05 + 1e-3).to(cuda_dev)
    tw = TernaryWeights(W, k.pack_ternary(W), torch.tensor([2.0 ** -6], device=cuda_dev))
    expect_int8 = (M, N, K) == (16384, 768, 1536)
    assert _pair_kernel_wins(M, N, K, A.device) == expect_int8
    got = ternary_matmul(A, tw, xs)
    ref = k.bitlinear_packed(A, tw.w2, xs, tw.scale)
    _eq(got, ref, f"ternary_matmul {M}x{N}x{K}")


def test_gemm_packed_config3_slice(cuda_dev):
    """Config-3 inputs with the weights packed 2 bits each: a 1024-row slice."""
    from mamba_integer_b200 import synth
    k = _mi()
    A, a_scale, Wq, ws = synth.bitlinear_inputs(M=1024, K=2048, N=1024)
    Wp = k.pack_ternary(Wq.to(cuda_dev))
    ref = orc.gemm_i8_i32(A.numpy(), Wq.numpy())
    _eq(k.bitlinear_packed(A.to(cuda_dev), Wp), ref, "config-3 slice, packed weights")


def test_gemm_packed_rejects_k_not_multiple_of_64(cuda_dev):
    from mamba_integer_b200 import _lib
    k = _mi()
    A = torch.zeros(128, 48, dtype=torch.int8, device=cuda_dev)
    Wp = torch.zeros(32, 12, dtype=torch.uint8, device=cuda_dev)
    with pytest.raises(_lib.MIError, match="status -2"):
        k.bitlinear_packed(A, Wp)


# ---------------------------------------------------------------- conv / ssm / element-wise
@pytest.mark.parametrize("bsz,L,D", [(2, 37, 512), (1, 130, 1536), (3, 67, 100), (1, 5, 4096)])
def test_conv_act_quant_matches_oracle(cuda_dev, bsz, L, D):
    k = _mi()
    g = torch.Generator().manual_seed(L + D)
    xz = torch.randn(bsz * L, 2 * D, generator=g) * 20
    w = torch.rand(D, 1, 4, generator=g) - 0.5
    b = torch.rand(D, generator=g) - 0.5
    _, act_ref = orc.conv_sqp(xz[:, :D].reshape(bsz, L, D).numpy(), w.numpy(), b.numpy())
    act_ref = act_ref.reshape(bsz * L, D)
    q_ref, s_ref = orc.quant_rows(act_ref)
    act, xq, xs = k.conv_act_quant(xz.to(cuda_dev), w.to(cuda_dev), b.to(cuda_dev), bsz, L, D)
    _eq(act, act_ref, "act")
    _eq(xq, q_ref, "xq")
    _eq(xs, s_ref, "xscale")
    act, xq, xs = k.conv_act_quant_rows(xz.to(cuda_dev), w.to(cuda_dev), b.to(cuda_dev), bsz, L, D)
    _eq(act, act_ref, "act (row kernel)")
    _eq(xq, q_ref, "xq (row kernel)")
    _eq(xs, s_ref, "xscale (row kernel)")


@pytest.mark.parametrize("bsz,L,D,R", [(2, 70, 512, 16), (1, 300, 1536, 48), (3, 5, 160, 16)])
def test_ssm_scan_matches_oracle(cuda_dev, bsz, L, D, R):
    k = _mi()
    g = torch.Generator().manual_seed(bsz + L + D)
    T = bsz * L
    act = torch.rand(T, D, generator=g) * 5
    xp = torch.randn(T, R + 32, generator=g) * 2
    modraw = torch.randn(T, D, generator=g) * 15
    modraw[::7, ::5] = 1e9  # ste_clamp rounding edge
    z = torch.randn(T, 2 * D, generator=g) * 3
    base = torch.randint(29492, 32736, (D, 16), generator=g).float()
    base[0, :] = 31990.0  # base + mod crosses 32000
    base[1, :] = 5.0      # base + mod crosses 0
    y_ref = orc.ssm(act.numpy(), np.ascontiguousarray(xp[:, R:].numpy()), modraw.numpy(),
                    np.ascontiguousarray(z[:, D:].numpy()), base.numpy(), bsz, L)
    dv = lambda t: t.to(cuda_dev)  # noqa: E731
    xpd, zd = dv(xp), dv(z)
    amax = torch.zeros(T, device=cuda_dev)
    y = k.ssm_scan(dv(act), xpd[:, R:], dv(modraw), zd[:, D:], dv(base), bsz, L, amax=amax)
    _eq(y, y_ref, "ssm y")
    _eq(amax, np.abs(y_ref).max(axis=1), "row absmax")


@pytest.mark.parametrize("bases", ["wide", "below_clamp"])
@pytest.mark.parametrize("split", [1, 2, 3, 4, 8, 0])
@pytest.mark.parametrize("bsz,L,D,R", [(2, 70, 512, 16), (1, 300, 1536, 48), (2, 9, 96, 64), (1, 33, 72, 20)])
def test_ssm_scan_fused_dt_matches_oracle(cuda_dev, bsz, L, D, R, split, bases):
    """dt_proj fused into the scan: same result as quantise -> BitLinear -> scan.
    bases "wide": the decay clamp at 32000 binds for some states, and the last
    channel group takes the step-by-step path; "below_clamp": every base <= 31964
    (the model initialises them at 16384), where the clamp never binds."""
    k = _mi()
    g = torch.Generator().manual_seed(5 * bsz + L + D + R)
    T = bsz * L
    R16 = (R + 15) // 16 * 16
    act = torch.rand(T, D, generator=g) * 5
    xp = torch.randn(T, R + 32, generator=g) * 2
    z = torch.randn(T, 2 * D, generator=g) * 3
    if bases == "wide":
        base = torch.randint(29492, 32736, (D, 16), generator=g).float()
        base[0, :] = 31990.0  # base + mod crosses 32000
        base[D - 1, :3] = 5.0  # base + mod crosses 0: the step-by-step path for the last channel group
    else:
        base = torch.randint(37, 31965, (D, 16), generator=g).float()
        base[0, :] = 31964.0  # the largest base without the clamp
        base[1, :] = 16384.0
    wdt = torch.randint(-1, 2, (D, R), generator=g, dtype=torch.int8)
    ws = np.float32(2.0 ** -5)
    dtq, dts = orc.quant_rows(np.ascontiguousarray(xp[:, :R].numpy()))
    modraw = orc.bitlinear(dtq, dts, wdt.numpy(), ws)
    y_ref, h_ref = orc.ssm(act.numpy(), np.ascontiguousarray(xp[:, R:].numpy()), modraw,
                           np.ascontiguousarray(z[:, D:].numpy()), base.numpy(), bsz, L, want_h=True)
    dv = lambda t: t.to(cuda_dev)  # noqa: E731
    dtq_d = torch.zeros(T, R16, dtype=torch.int8, device=cuda_dev)
    dts_d = torch.empty(T, device=cuda_dev)
    xpd, zd = dv(xp), dv(z)
    k.quantize_rows(xpd, K=R, out=dtq_d, xscale=dts_d)
    w16 = torch.zeros(D, R16, dtype=torch.int8)
    w16[:, :R] = wdt
    amax = torch.zeros(T, device=cuda_dev)
    h_out = torch.full((bsz, D, 16), 7.0, device=cuda_dev)
    y = k.ssm_scan_dt(dv(act), xpd[:, R:], dtq_d, dts_d, dv(w16), dv(torch.tensor([ws])), R, zd[:, D:], dv(base),
                      bsz, L, amax=amax, split=split, h_out=h_out)
    _eq(y, y_ref, "fused-dt ssm y")
    _eq(amax, np.abs(y_ref).max(axis=1), "row absmax")
    _eq(h_out, h_ref, "final states")


def test_scan_convex_and_elementwise_match_reference_fixtures(cuda_dev):
    import os
    k = _mi()
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "stages.npz"))
    u, nums = cases.scan_inputs()
    _eq(k.scan_convex(torch.from_numpy(u).to(cuda_dev), torch.from_numpy(nums).to(cuda_dev)), gold["scan.h"], "scan")
    e = torch.from_numpy(cases.edge_values()).to(cuda_dev)
    _eq(k.squareplus_clamp(e, -50.0, 50.0), gold["sqp.y"], "squareplus")
    _eq(k.ste_clamp(e, -20.0, 20.0), gold["ste20.y"], "ste_clamp")
    _eq(k.ste_clamp(e, 0.0, 32000.0), gold["ste_dec.y"], "ste_clamp decay")
    y, z = cases.gate_inputs()
    _eq(k.sigmoid_gate(torch.from_numpy(y).to(cuda_dev), torch.from_numpy(z).to(cuda_dev)), gold["gate.y"], "gate")
    q, s = k.quantize_rows(torch.from_numpy(cases.quant_inputs()).to(cuda_dev))
    _eq(q, gold["quant.xq"], "quant")
    _eq(s, gold["quant.scale"], "quant scale")
