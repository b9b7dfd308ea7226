"""torch-tensor wrappers over the C ABI (one function per kernel entry point).

Every wrapper checks devices/dtypes/contiguity, allocates its outputs with
torch (the C ABI never allocates), launches on the current CUDA stream and
raises on a non-zero status.  The names the reference's model imports from
its Triton package are provided as aliases at the bottom
(src/triton_kernels/bitnet_kernels.py:98, :295; dyadic_scan.py:462;
fused_activations.py:229, :399, :511).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, dtype, name: str, contiguous: bool = True):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _scalar_dev(v, like: torch.Tensor) -> torch.Tensor:
    if isinstance(v, torch.Tensor):
        return v.to(device=like.device, dtype=torch.float32).reshape(1).contiguous()
    return torch.tensor([float(v)], dtype=torch.float32, device=like.device)


# ---------------------------------------------------------------------------
# integer dyadic scan
# ---------------------------------------------------------------------------
def scan_i32(x: torch.Tensor, B: torch.Tensor, C: torch.Tensor, n: torch.Tensor, k: int = 15,
             h0: Optional[torch.Tensor] = None, y_dtype=torch.int32, check_errors: bool = True
             ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Integer selective scan; returns (y [b,L,D] y_dtype, h_T [b,D,N] int32)."""
    for t, nm in ((x, "x"), (B, "B"), (C, "C"), (n, "n")):
        _need(t, torch.int32, nm)
    bsz, L, D = x.shape
    N = n.shape[1]
    if B.shape != (bsz, L, N) or C.shape != (bsz, L, N) or n.shape != (D, N):
        raise ValueError("shape mismatch between x, B, C and n")
    h = torch.zeros(bsz, D, N, dtype=torch.int32, device=x.device) if h0 is None else h0.clone()
    _need(h, torch.int32, "h0")
    y = torch.empty(bsz, L, D, dtype=y_dtype, device=x.device)
    y32 = y if y_dtype == torch.int32 else None
    y64 = y if y_dtype == torch.int64 else None
    if y32 is None and y64 is None:
        raise TypeError("y_dtype must be torch.int32 or torch.int64")
    lib = _lib.load()
    _lib.check(lib.mi_scan_i32(x.data_ptr(), B.data_ptr(), C.data_ptr(), n.data_ptr(), int(k), _ptr(y32), _ptr(y64),
                               h.data_ptr(), bsz, L, D, N, _stream()), "mi_scan_i32")
    if check_errors:
        err = _lib.device_error(_stream())
        if err:
            raise OverflowError(f"integer scan device error word {err:#x} "
                                "(1 = int32 overflow, 4 = input outside the stated range)")
    return y, h


# ---------------------------------------------------------------------------
# row stages
# ---------------------------------------------------------------------------
def bitshift_norm(x: torch.Tensor, gamma: torch.Tensor, step, center_once: bool = False
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """BitShiftNorm forward (reference CPU semantics): returns (y, inv_rms[rows]).
    center_once gives BitShiftNormFunction.forward alone (its input already centred once)."""
    _need(x, torch.float32, "x")
    D = x.shape[-1]
    T = x.numel() // D
    y = torch.empty_like(x)
    inv = torch.empty(T, dtype=torch.float32, device=x.device)
    g = gamma.detach().to(torch.float32).contiguous()
    s = _scalar_dev(step, x)
    _lib.check(_lib.load().mi_bitshift_norm(x.data_ptr(), g.data_ptr(), s.data_ptr(), y.data_ptr(), inv.data_ptr(),
                                            T, D, int(center_once), _stream()), "mi_bitshift_norm")
    return y, inv


def quantize_rows(x: torch.Tensor, K: Optional[int] = None, out: Optional[torch.Tensor] = None,
                  xscale: Optional[torch.Tensor] = None, amax: Optional[torch.Tensor] = None,
                  clear: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row absmax int8 quantisation of the first K columns of a 2-D fp32
    tensor (row stride taken from x); returns (xq int8 [T, ldq], x_scale [T]).
    ``clear`` (fp32 [T], optional) is zero-filled on the way (the row maxima
    the fused scan accumulates next)."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D with unit column stride")
    _need(x, torch.float32, "x", contiguous=False)
    T, W = x.shape
    K = W if K is None else K
    if out is None:
        out = torch.empty(T, K, dtype=torch.int8, device=x.device)
    if xscale is None:
        xscale = torch.empty(T, dtype=torch.float32, device=x.device)
    if clear is not None:
        _need(clear, torch.float32, "clear")
        if clear.numel() < T:
            raise ValueError("clear must hold one float per row")
    _lib.check(_lib.load().mi_quantize_rows(x.data_ptr(), x.stride(0), T, K, out.data_ptr(), out.stride(0),
                                            xscale.data_ptr(), _ptr(amax), _ptr(clear), _stream()),
               "mi_quantize_rows")
    return out, xscale


def quantize_activations(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """activation_quant_dynamic: returns (xq as fp32 integer values [..., K],
    scale / 127 [..., 1]) like the reference."""
    K = x.shape[-1]
    q, s = quantize_rows(x.contiguous().view(-1, K))
    return q.to(torch.float32).view_as(x), s.view(*x.shape[:-1], 1)


def rowprep(gamma, step, T: int, D: int, x=None, delta=None, res_gate=None, ids=None, emb=None, x_out=None,
            y_norm=None, xq=None, xscale=None) -> None:
    """Fused residual update + BitShiftNorm + int8 quantisation (see mi_rowprep)."""
    vocab = emb.shape[0] if emb is not None else 0
    _lib.check(_lib.load().mi_rowprep(_ptr(x), _ptr(delta), _ptr(res_gate), _ptr(ids), _ptr(emb), vocab, _ptr(x_out),
                                      gamma.data_ptr(), step.data_ptr(), _ptr(y_norm), _ptr(xq), _ptr(xscale), T, D,
                                      _stream()), "mi_rowprep")


# ---------------------------------------------------------------------------
# BitLinear GEMM
# ---------------------------------------------------------------------------
def bitlinear_i8(A: torch.Tensor, W: torch.Tensor, a_scale: Optional[torch.Tensor] = None,
                 w_scale: Optional[torch.Tensor] = None, out_scale: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, K: Optional[int] = None) -> torch.Tensor:
    """tcgen05 int8 GEMM: A int8 [M, >=K] (row stride from A), W int8 [N, K].
    With a_scale/w_scale: fp32 acc * (w_scale * a_scale[m]) [* out_scale];
    without: the int32 accumulators."""
    _need(W, torch.int8, "W")
    if A.dim() != 2 or A.stride(1) != 1:
        raise ValueError("A must be 2-D with unit column stride")
    _need(A, torch.int8, "A", contiguous=False)
    M = A.shape[0]
    N, Kw = W.shape
    K = Kw if K is None else K
    scaled = a_scale is not None
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32 if scaled else torch.int32, device=A.device)
    epi = _lib.MI_EPI_F32_SCALED if scaled else _lib.MI_EPI_I32
    _lib.check(_lib.load().mi_bitlinear_i8(A.data_ptr(), A.stride(0), W.data_ptr(), _ptr(a_scale), _ptr(w_scale),
                                           _ptr(out_scale), out.data_ptr(), out.stride(0), M, N, K, epi, _stream()),
               "mi_bitlinear_i8")
    return out


def pack_ternary(W: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """int8 ternary weights [N, K] -> 2-bit packed [N, K/4] uint8 (on the GPU)."""
    _need(W, torch.int8, "W")
    N, K = W.shape
    if out is None:
        out = torch.empty(N, K // 4, dtype=torch.uint8, device=W.device)
    _lib.check(_lib.load().mi_pack_ternary(W.data_ptr(), W.stride(0), out.data_ptr(), N, K, _stream()),
               "mi_pack_ternary")
    return out


def bitlinear_packed(A: torch.Tensor, Wp: torch.Tensor, a_scale: Optional[torch.Tensor] = None,
                     w_scale: Optional[torch.Tensor] = None, out_scale: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None, K: Optional[int] = None) -> torch.Tensor:
    """bitlinear_i8 with 2-bit packed weights Wp uint8 [N, K/4] (see pack_ternary)."""
    _need(Wp, torch.uint8, "Wp")
    if A.dim() != 2 or A.stride(1) != 1:
        raise ValueError("A must be 2-D with unit column stride")
    _need(A, torch.int8, "A", contiguous=False)
    M = A.shape[0]
    N = Wp.shape[0]
    K = 4 * Wp.shape[1] if K is None else K
    scaled = a_scale is not None
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32 if scaled else torch.int32, device=A.device)
    epi = _lib.MI_EPI_F32_SCALED if scaled else _lib.MI_EPI_I32
    _lib.check(_lib.load().mi_bitlinear_packed(A.data_ptr(), A.stride(0), Wp.data_ptr(), _ptr(a_scale),
                                               _ptr(w_scale), _ptr(out_scale), out.data_ptr(), out.stride(0), M, N,
                                               K, epi, _stream()),
               "mi_bitlinear_packed")
    return out


# ---------------------------------------------------------------------------
# conv / scan / element-wise
# ---------------------------------------------------------------------------
def bitlinear_packed_norm_sqp(A: torch.Tensor, Wp: torch.Tensor, a_scale: torch.Tensor, w_scale: torch.Tensor,
                              gamma: torch.Tensor, step: torch.Tensor, acc: Optional[torch.Tensor] = None,
                              out: Optional[torch.Tensor] = None, stats_ws: Optional[torch.Tensor] = None
                              ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Config 3's BitLinear + BitShift norm + squareplus (mi_bitlinear_packed_norm_sqp):
    returns (acc int32 [M, N], out fp32 [M, N]).  stats_ws: int64 [M, 2] workspace."""
    _need(Wp, torch.uint8, "Wp")
    if A.dim() != 2 or A.stride(1) != 1:
        raise ValueError("A must be 2-D with unit column stride")
    _need(A, torch.int8, "A", contiguous=False)
    for t, nm in ((a_scale, "a_scale"), (w_scale, "w_scale"), (gamma, "gamma"), (step, "step")):
        _need(t, torch.float32, nm)
    M, N, K = A.shape[0], Wp.shape[0], 4 * Wp.shape[1]
    if acc is None:
        acc = torch.empty(M, N, dtype=torch.int32, device=A.device)
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=A.device)
    if stats_ws is None:
        stats_ws = torch.empty(M, 2, dtype=torch.int64, device=A.device)
    _need(acc, torch.int32, "acc", contiguous=False)
    _need(out, torch.float32, "out", contiguous=False)
    _need(stats_ws, torch.int64, "stats_ws")
    _lib.check(_lib.load().mi_bitlinear_packed_norm_sqp(A.data_ptr(), A.stride(0), Wp.data_ptr(), a_scale.data_ptr(),
                                                        w_scale.data_ptr(), gamma.data_ptr(), step.data_ptr(),
                                                        acc.data_ptr(), acc.stride(0), out.data_ptr(), out.stride(0),
                                                        stats_ws.data_ptr(), M, N, K, _stream()),
               "mi_bitlinear_packed_norm_sqp")
    return acc, out


def conv_act_quant(xz: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, batch: int, L: int, D: int,
                   act=None, xq=None, xscale=None, quantize: bool = True, amax_ws=None):
    """Causal depthwise conv + ste_clamp + squareplus (+ int8 quantisation) of
    the first D columns of xz [batch*L, ldx]."""
    T = batch * L
    if act is None:
        act = torch.empty(T, D, dtype=torch.float32, device=xz.device)
    if quantize:
        if xq is None:
            xq = torch.empty(T, D, dtype=torch.int8, device=xz.device)
        if xscale is None:
            xscale = torch.empty(T, dtype=torch.float32, device=xz.device)
        if amax_ws is None:
            amax_ws = torch.empty(T, dtype=torch.float32, device=xz.device)
    wc = w.detach().to(torch.float32).reshape(D, 4).contiguous()
    bc = bias.detach().to(torch.float32).contiguous()
    _lib.check(_lib.load().mi_conv_act_quant(xz.data_ptr(), xz.stride(0), wc.data_ptr(), bc.data_ptr(),
                                             act.data_ptr(), _ptr(xq), _ptr(xscale), _ptr(amax_ws), batch, L, D,
                                             _stream()),
               "mi_conv_act_quant")
    return act, xq, xscale


def conv_act_quant_rows(xz: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, batch: int, L: int, D: int,
                        act=None, xq=None, xscale=None):
    """conv_act_quant in one row-owning kernel (mi_conv_act_quant_rows): same
    results, no workspace."""
    T = batch * L
    if act is None:
        act = torch.empty(T, D, dtype=torch.float32, device=xz.device)
    if xq is None:
        xq = torch.empty(T, D, dtype=torch.int8, device=xz.device)
    if xscale is None:
        xscale = torch.empty(T, dtype=torch.float32, device=xz.device)
    wc = w.detach().to(torch.float32).reshape(D, 4).contiguous()
    bc = bias.detach().to(torch.float32).contiguous()
    _lib.check(_lib.load().mi_conv_act_quant_rows(xz.data_ptr(), xz.stride(0), wc.data_ptr(), bc.data_ptr(),
                                                  act.data_ptr(), xq.data_ptr(), xscale.data_ptr(), batch, L, D,
                                                  _stream()),
               "mi_conv_act_quant_rows")
    return act, xq, xscale


def ssm_scan(act, bc, modraw, z, base, batch: int, L: int, y=None, amax=None):
    """Fused selective scan + gate (see mi_ssm_scan).  bc / z may be column
    slices (row stride taken from the tensor)."""
    D, N = base.shape
    T = batch * L
    if y is None:
        y = torch.empty(T, D, dtype=torch.float32, device=act.device)
    _lib.check(_lib.load().mi_ssm_scan(act.data_ptr(), bc.data_ptr(), bc.stride(0), modraw.data_ptr(), z.data_ptr(),
                                       z.stride(0), base.data_ptr(), y.data_ptr(), _ptr(amax), batch, L, D, N,
                                       _stream()), "mi_ssm_scan")
    return y


def ssm_scan_dt(act, bc, dtq, dts, w_dt, w_dt_scale, R: int, z, base, batch: int, L: int, y=None, amax=None,
                split: int = 0, h_out=None):
    """ssm_scan with dt_proj fused (see mi_ssm_scan_dt): dtq int8 [T, ldq] quantised
    dt rows, dts [T] their scales, w_dt int8 [D, ceil16(R)], w_dt_scale [1].
    split: kernel variant (1/2/4/8 lanes per channel, 3 = pipelined (four warps),
    0 = automatic); h_out [batch, D, N]: final states."""
    D, N = base.shape
    T = batch * L
    if y is None:
        y = torch.empty(T, D, dtype=torch.float32, device=act.device)
    _lib.check(_lib.load().mi_ssm_scan_dt(act.data_ptr(), bc.data_ptr(), bc.stride(0), dtq.data_ptr(), dtq.stride(0),
                                          dts.data_ptr(), w_dt.data_ptr(), w_dt_scale.data_ptr(), R, z.data_ptr(),
                                          z.stride(0), base.data_ptr(), y.data_ptr(), _ptr(amax), _ptr(h_out), batch,
                                          L, D, N, int(split), _stream()), "mi_ssm_scan_dt")
    return y


# ---------------------------------------------------------------------------
# decode steps
# ---------------------------------------------------------------------------
def conv_step(xz: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, win: torch.Tensor, D: int, xq: torch.Tensor,
              xscale: torch.Tensor, act: Optional[torch.Tensor] = None):
    """One causal-conv position per stream: xz rows [batch, >=D] (x_t = first D
    columns), win [batch, 3, D] advanced in place; writes act (optional), xq, xscale."""
    batch = xz.shape[0]
    _lib.check(_lib.load().mi_conv_step(xz.data_ptr(), xz.stride(0), w.data_ptr(), bias.data_ptr(), win.data_ptr(),
                                        _ptr(act), xq.data_ptr(), xscale.data_ptr(), batch, D, _stream()),
               "mi_conv_step")


def ssm_step(act, xp, R: int, w_dt, w_dt_scale, z, base, h, xq, xscale, y=None):
    """One selective-scan position per stream (see mi_ssm_step); h [batch, D, 16]
    is updated in place; writes y (optional), xq, xscale."""
    batch, D = act.shape
    N = base.shape[1]
    _lib.check(_lib.load().mi_ssm_step(act.data_ptr(), xp.data_ptr(), xp.stride(0), R, w_dt.data_ptr(),
                                       w_dt_scale.data_ptr(), z.data_ptr(), z.stride(0), base.data_ptr(), h.data_ptr(),
                                       _ptr(y), xq.data_ptr(), xscale.data_ptr(), batch, D, N, _stream()),
               "mi_ssm_step")


def decode_mid(xz, conv_w, conv_b, win, w_x, w_x_scale, R: int, w_dt, w_dt_scale, base, h, xq, xscale,
               xp_out=None):
    """conv step + x_proj + scan step + gate + quantisation for one decode
    position (see mi_decode_mid); win and h advance in place."""
    batch = xz.shape[0]
    D, N = base.shape
    _lib.check(_lib.load().mi_decode_mid(xz.data_ptr(), xz.stride(0), conv_w.data_ptr(), conv_b.data_ptr(),
                                         win.data_ptr(), w_x.data_ptr(), w_x_scale.data_ptr(), R, w_dt.data_ptr(),
                                         w_dt_scale.data_ptr(), base.data_ptr(), h.data_ptr(), _ptr(xp_out),
                                         xq.data_ptr(), xscale.data_ptr(), batch, D, N, _stream()),
               "mi_decode_mid")


def decode_mid_packed(xz, conv_w, conv_b, win, w_x_packed, w_x_scale, R: int, w_dt, w_dt_scale, base, h, xq, xscale,
                      xp_out=None):
    """decode_mid with the x_proj weights in the 2-bit packed form (pack_ternary,
    uint8 [R + 2N, D/4]); see mi_decode_mid_packed.  D % 64 == 0."""
    batch = xz.shape[0]
    D, N = base.shape
    _need(w_x_packed, torch.uint8, "w_x_packed")
    if tuple(w_x_packed.shape) != (R + 2 * N, D // 4) or not w_x_packed.is_contiguous():
        raise ValueError(f"w_x_packed must be contiguous [{R + 2 * N}, {D // 4}]")
    _lib.check(_lib.load().mi_decode_mid_packed(xz.data_ptr(), xz.stride(0), conv_w.data_ptr(), conv_b.data_ptr(),
                                                win.data_ptr(), w_x_packed.data_ptr(), w_x_scale.data_ptr(), R,
                                                w_dt.data_ptr(), w_dt_scale.data_ptr(), base.data_ptr(), h.data_ptr(),
                                                _ptr(xp_out), xq.data_ptr(), xscale.data_ptr(), batch, D, N,
                                                _stream()),
               "mi_decode_mid_packed")


def argmax_rows(x: torch.Tensor, V: Optional[int] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """torch.argmax(x[:, :V], dim=-1) as int64 (first index of the maximum, NaN highest)."""
    T = x.shape[0]
    V = x.shape[1] if V is None else V
    if out is None:
        out = torch.empty(T, dtype=torch.int64, device=x.device)
    _lib.check(_lib.load().mi_argmax_rows(x.data_ptr(), x.stride(0), T, V, out.data_ptr(), _stream()),
               "mi_argmax_rows")
    return out


def scan_convex(u: torch.Tensor, nums: torch.Tensor) -> torch.Tensor:
    _need(u, torch.float32, "u")
    _need(nums, torch.float32, "nums")
    b, L, DN = u.shape
    h = torch.empty_like(u)
    _lib.check(_lib.load().mi_scan_convex(u.data_ptr(), nums.data_ptr(), h.data_ptr(), b, L, DN, _stream()),
               "mi_scan_convex")
    return h


def squareplus_clamp(x: torch.Tensor, low: float = -50.0, high: float = 50.0) -> torch.Tensor:
    _need(x, torch.float32, "x")
    y = torch.empty_like(x)
    _lib.check(_lib.load().mi_squareplus_clamp(x.data_ptr(), y.data_ptr(), x.numel(), low, high, _stream()),
               "mi_squareplus_clamp")
    return y


def ste_clamp(x: torch.Tensor, low: float, high: float) -> torch.Tensor:
    _need(x, torch.float32, "x")
    y = torch.empty_like(x)
    _lib.check(_lib.load().mi_ste_clamp(x.data_ptr(), y.data_ptr(), x.numel(), low, high, _stream()), "mi_ste_clamp")
    return y


def sigmoid_gate(y: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    _need(y, torch.float32, "y")
    _need(z, torch.float32, "z")
    o = torch.empty_like(y)
    _lib.check(_lib.load().mi_sigmoid_gate(y.data_ptr(), z.data_ptr(), o.data_ptr(), y.numel(), _stream()),
               "mi_sigmoid_gate")
    return o


# Names used by the reference model for its GPU kernels.
def fast_bitshift_norm(x, gamma, step_size=None):
    step = torch.ones(1, device=x.device) if step_size is None else step_size
    return bitshift_norm(x.contiguous(), gamma, step)


def scan_convex_backward(grad_h: torch.Tensor, h: torch.Tensor, u: torch.Tensor, nums: torch.Tensor
                         ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Backward of the convex dyadic scan (mi_scan_convex_backward): (grad_u, grad_nums)."""
    for t, nm in ((grad_h, "grad_h"), (h, "h"), (u, "u"), (nums, "nums")):
        _need(t, torch.float32, nm)
        if t.shape != grad_h.shape or t.dim() != 3:
            raise ValueError(f"{nm} must be [batch, L, DN] like grad_h")
    B, L, DN = grad_h.shape
    gu = torch.empty_like(grad_h)
    gn = torch.empty_like(grad_h)
    _lib.check(_lib.load().mi_scan_convex_backward(grad_h.data_ptr(), h.data_ptr(), u.data_ptr(), nums.data_ptr(),
                                                   gu.data_ptr(), gn.data_ptr(), B, L, DN, _stream()),
               "mi_scan_convex_backward")
    return gu, gn


def quant_ste_backward(grad_xq: torch.Tensor, amax: torch.Tensor) -> torch.Tensor:
    """Straight-through backward of the activation quantisation (mi_quant_ste_backward):
    grad_xq [T, K], amax [T] (each row's max |x|) -> grad_x [T, K]."""
    _need(grad_xq, torch.float32, "grad_xq")
    _need(amax, torch.float32, "amax")
    T, K = grad_xq.shape
    if amax.numel() != T:
        raise ValueError("amax must hold one value per row")
    gx = torch.empty_like(grad_xq)
    _lib.check(_lib.load().mi_quant_ste_backward(grad_xq.data_ptr(), amax.data_ptr(), gx.data_ptr(), T, K, _stream()),
               "mi_quant_ste_backward")
    return gx


class QuantizeActivationsFunction(torch.autograd.Function):
    """Activation quantisation with the reference's straight-through backward
    (src/triton_kernels/bitnet_kernels.py:48-95): forward (xq as fp32 integer
    values, amax / 127); backward clamp(grad * 127 / clamp(amax, min=0.01), +-100)."""

    @staticmethod
    def forward(ctx, x):
        K = x.shape[-1]
        x2 = x.detach().float().contiguous().view(-1, K)
        # the row maximum the backward needs (the reference saves max(amax, 1e-8) itself,
        # which amax / 127 does not give back exactly); a maximum is exact in any order
        amax = x2.abs().amax(-1).clamp(min=1e-8).contiguous()
        q, s = quantize_rows(x2, amax=amax)
        ctx.save_for_backward(amax)
        ctx.original_shape = x.shape
        return q.to(torch.float32).view(x.shape), s.view(*x.shape[:-1], 1)

    @staticmethod
    def backward(ctx, grad_x_quant, grad_scale):
        (amax,) = ctx.saved_tensors
        K = ctx.original_shape[-1]
        g = grad_x_quant.float().contiguous().view(-1, K)
        return quant_ste_backward(g, amax).view(ctx.original_shape)


def fast_quantize_activations(x):
    """Triton-name wrapper of the reference (src/triton_kernels/bitnet_kernels.py:98):
    quantisation with the straight-through backward."""
    return QuantizeActivationsFunction.apply(x)


fused_squareplus_clamp = squareplus_clamp
fused_ste_clamp = ste_clamp
fused_sigmoid_gate = sigmoid_gate


def dyadic_scan_triton_fast(u, nums):
    return scan_convex(u.contiguous(), nums.contiguous())
