// ssm.cu -- the selective-scan half of MambaIntegerBlock on sm_100a:
//   * causal depthwise conv + ste_clamp + squareplus + int8 quantisation
//     (feeds x_proj and the scan), one warp per token row;
//   * the fused selective scan: decay clamp, dt, u = (x*dt)*B, the convex
//     dyadic recurrence, y = sum_n h*C and the algebraic-sigmoid gate, one
//     thread per (sequence, channel) carrying its 16 fp32 states in registers;
//   * the stand-alone convex scan on materialised u / nums and the
//     element-wise ops of the Triton wrappers.
//
// Arithmetic follows the reference CPU path operation by operation (see
// mi_common.cuh); the FMAs used are exactly the reference's own: bias-first
// tap accumulation of the conv and the n-ascending accumulation of h.C.
#include "mi_common.cuh"

namespace mi {
namespace ssm {

// ---------------------------------------------------------------------------
// conv + activation + quantisation
// ---------------------------------------------------------------------------
// xz: [batch*L, ldx], conv input = columns [0, D).  act/xq: [batch*L, D].
__global__ void __launch_bounds__(256)
conv_act_quant_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ w,
                      const float* __restrict__ bias, float* __restrict__ act, int8_t* __restrict__ xq,
                      float* __restrict__ xscale, int L, int D, int T) {
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
        const int t = row % L;  // position within its sequence
        float am = 0.0f;
        bool nan = false;
        for (int c = lane; c < D; c += 32) {
            const float4 wc = *reinterpret_cast<const float4*>(w + 4 * c);
            const float wk[4] = {wc.x, wc.y, wc.z, wc.w};
            float acc = bias[c];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int dt = 3 - k;  // tap k reads position t - 3 + k
                const float xv = (t - dt >= 0) ? xz[(size_t)(row - dt) * ldx + c] : 0.0f;
                acc = __fmaf_rn(wk[k], xv, acc);
            }
            const float a = squareplus(ste_clamp(acc, -50.0f, 50.0f));
            act[(size_t)row * D + c] = a;
            const float aa = fabsf(a);
            nan |= (aa != aa);
            am = fmaxf(am, aa);
        }
        if (xq) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
            nan = __any_sync(0xffffffffu, nan);
            const float amax = nan ? __int_as_float(0x7fc00000) : am;
            const float sc = clamp_t(amax, 1e-8f, __int_as_float(0x7f800000));
            const float inv = __fmul_rn(__frcp_rn(sc), 127.0f);
            // each lane re-reads only the values it wrote itself
            for (int c = lane; c < D; c += 32)
                xq[(size_t)row * D + c] = (int8_t)quant_i8(__fmul_rn(act[(size_t)row * D + c], inv));
            if (lane == 0) xscale[row] = __fdiv_rn(sc, 127.0f);
        }
    }
}

// ---------------------------------------------------------------------------
// fused selective scan
// ---------------------------------------------------------------------------
constexpr int NS = 16;
constexpr int SCAN_THREADS = 128;
constexpr int TC = 32;  // time steps of B/C staged per chunk

__global__ void __launch_bounds__(SCAN_THREADS)
ssm_scan_kernel(const float* __restrict__ act, const float* __restrict__ bc, int ldbc,
                const float* __restrict__ modraw, const float* __restrict__ z, int ldz,
                const float* __restrict__ base, float* __restrict__ y, float* __restrict__ amax, int L, int D) {
    __shared__ float sbc[TC][2 * NS];
    const int b = blockIdx.y;
    const int d = blockIdx.x * SCAN_THREADS + threadIdx.x;
    const bool active = d < D;
    const int dd = active ? d : 0;

    float bn[NS], h[NS];
    float bmin = __int_as_float(0x7f800000), bmax = -__int_as_float(0x7f800000);
#pragma unroll
    for (int n = 0; n < NS; n++) {
        bn[n] = base[(size_t)dd * NS + n];
        h[n] = 0.0f;
        bmin = fminf(bmin, bn[n]);
        bmax = fmaxf(bmax, bn[n]);
    }
    bool bnan = false;
#pragma unroll
    for (int n = 0; n < NS; n++) bnan |= (bn[n] != bn[n]);

    const size_t row0 = (size_t)b * L;
    for (int t0 = 0; t0 < L; t0 += TC) {
        const int tn = min(TC, L - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < tn * 2 * NS; i += SCAN_THREADS) {
            const int r = i / (2 * NS), q = i % (2 * NS);
            sbc[r][q] = bc[(row0 + t0 + r) * ldbc + q];
        }
        __syncthreads();
        if (!active) continue;
        for (int r = 0; r < tn; r++) {
            const size_t row = row0 + t0 + r;
            const float xa = act[row * D + d];
            const float mr = modraw[row * D + d];
            const float zz = z[row * ldz + d];
            // decay_mod = ste_clamp(dt_proj(dt), -20, 20)           (:419-422)
            const float mod = ste_clamp(mr, -20.0f, 20.0f);
            // dt_val = ste_clamp(squareplus(decay_mod) * 0.01, 1e-3, 0.1)  (:427)
            const float dtv = ste_clamp(__fmul_rn(squareplus(mod), 0.01f), 0.001f, 0.1f);
            // u = (x * dt_val) * B                                   (:428)
            const float xdt = __fmul_rn(xa, dtv);
            // decay_nums = ste_clamp(base + decay_mod, 0, 32000)    (:424).  When every
            // base + mod of this channel is strictly inside (0, 32000) the clamp is the
            // identity (rounding is monotone, so checking the extremes suffices).
            const bool inside = !bnan && (__fadd_rn(bmin, mod) > 0.0f) && (__fadd_rn(bmax, mod) <= 32000.0f);
            float yacc = 0.0f;
            if (inside) {
#pragma unroll
                for (int n = 0; n < NS; n++) {
                    const float num = __fadd_rn(bn[n], mod);
                    const float dec = __fmul_rn(num, 3.0517578125e-05f);  // num / 2^15, exact
                    const float u = __fmul_rn(xdt, sbc[r][n]);
                    // h = h * decay + (1 - decay) * u             (:309)
                    h[n] = __fadd_rn(__fmul_rn(h[n], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                }
            } else {
#pragma unroll
                for (int n = 0; n < NS; n++) {
                    const float num = ste_clamp(__fadd_rn(bn[n], mod), 0.0f, 32000.0f);
                    const float dec = __fmul_rn(num, 3.0517578125e-05f);
                    const float u = __fmul_rn(xdt, sbc[r][n]);
                    h[n] = __fadd_rn(__fmul_rn(h[n], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                }
            }
            // y = matmul(h, C[..., None]): FMA over n = 0..15 from 0    (:440)
#pragma unroll
            for (int n = 0; n < NS; n++) yacc = __fmaf_rn(h[n], sbc[r][NS + n], yacc);
            const float out = sigmoid_gate(yacc, zz);
            y[row * D + d] = out;
            if (amax) {
                // non-negative floats order like their bit patterns; NaN bits sort above inf
                atomicMax(reinterpret_cast<unsigned int*>(amax) + row, __float_as_uint(fabsf(out)));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// stand-alone convex scan and element-wise ops
// ---------------------------------------------------------------------------
__global__ void scan_convex_kernel(const float* __restrict__ u, const float* __restrict__ nums,
                                   float* __restrict__ h, int batch, int L, int DN) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int b = blockIdx.y;
    if (c >= DN) return;
    float hv = 0.0f;
    for (int t = 0; t < L; t++) {
        const size_t o = ((size_t)b * L + t) * DN + c;
        const float dec = __fdiv_rn(nums[o], 32768.0f);
        hv = __fadd_rn(__fmul_rn(hv, dec), __fmul_rn(__fsub_rn(1.0f, dec), u[o]));
        h[o] = hv;
    }
}

__global__ void squareplus_clamp_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, float lo,
                                        float hi) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = squareplus(ste_clamp(x[i], lo, hi));
}
__global__ void ste_clamp_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, float lo, float hi) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = ste_clamp(x[i], lo, hi);
}
__global__ void sigmoid_gate_kernel(const float* __restrict__ yv, const float* __restrict__ z, float* __restrict__ o,
                                    int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        o[i] = sigmoid_gate(yv[i], z[i]);
}

static int ew_blocks(int64_t n) {
    int64_t b = (n + 255) / 256;
    if (b > 148 * 32) b = 148 * 32;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace ssm
}  // namespace mi

extern "C" int mi_conv_act_quant(const float* xz, int ldx, const float* w, const float* bias, float* act, int8_t* xq,
                                 float* xscale, int batch, int L, int D, void* stream) {
    if (!xz || !w || !bias || !act) return MI_ERR_INVALID;
    if ((xq == nullptr) != (xscale == nullptr)) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || D <= 0 || ldx < D) return MI_ERR_INVALID;
    if (((uintptr_t)w) & 15) return MI_ERR_INVALID;
    const int T = batch * L;
    int blocks = mi::cdiv(T, 8);
    if (blocks > 148 * 16) blocks = 148 * 16;
    mi::ssm::conv_act_quant_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(xz, ldx, w, bias, act, xq, xscale, L, D,
                                                                             T);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_ssm_scan(const float* act, const float* bc, int ldbc, const float* modraw, const float* z, int ldz,
                           const float* base, float* y, float* amax, int batch, int L, int D, int N, void* stream) {
    if (!act || !bc || !modraw || !z || !base || !y) return MI_ERR_INVALID;
    if (N != mi::ssm::NS) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || L <= 0 || D <= 0 || ldbc < 2 * N || ldz < D) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(D, mi::ssm::SCAN_THREADS), batch);
    mi::ssm::ssm_scan_kernel<<<grid, mi::ssm::SCAN_THREADS, 0, (cudaStream_t)stream>>>(act, bc, ldbc, modraw, z, ldz,
                                                                                       base, y, amax, L, D);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_scan_convex(const float* u, const float* nums, float* h, int batch, int L, int DN, void* stream) {
    if (!u || !nums || !h) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || DN <= 0) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(DN, 128), batch);
    mi::ssm::scan_convex_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(u, nums, h, batch, L, DN);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_squareplus_clamp(const float* x, float* y, int64_t n, float lo, float hi, void* stream) {
    if (!x || !y || n < 0) return MI_ERR_INVALID;
    if (n == 0) return MI_OK;
    mi::ssm::squareplus_clamp_kernel<<<mi::ssm::ew_blocks(n), 256, 0, (cudaStream_t)stream>>>(x, y, n, lo, hi);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_ste_clamp(const float* x, float* y, int64_t n, float lo, float hi, void* stream) {
    if (!x || !y || n < 0) return MI_ERR_INVALID;
    if (n == 0) return MI_OK;
    mi::ssm::ste_clamp_kernel<<<mi::ssm::ew_blocks(n), 256, 0, (cudaStream_t)stream>>>(x, y, n, lo, hi);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_sigmoid_gate(const float* y, const float* z, float* out, int64_t n, void* stream) {
    if (!y || !z || !out || n < 0) return MI_ERR_INVALID;
    if (n == 0) return MI_OK;
    mi::ssm::sigmoid_gate_kernel<<<mi::ssm::ew_blocks(n), 256, 0, (cudaStream_t)stream>>>(y, z, out, n);
    MI_CHECK_LAUNCH();
    return MI_OK;
}
