// rowops.cu -- row-wise stages: BitShiftNorm, per-token int8 quantisation and
// the fused row pre-pass (residual update + norm + quantisation) that feeds
// every BitLinear whose input is the residual stream.
//
// One warp owns one row.  Lane a holds the elements a, a+32, a+64, ... of the
// row in registers, which is exactly the accumulator assignment of ATen's CPU
// cascade sum for an fp32 row with 8-lane vectors and 4-way ILP: element
// 32r + a goes to ILP slot a/8, vector lane a%8.  Each lane therefore folds
// its own values in the reference order, and the cross-lane combine replays
// ATen's fixed epilogue (slots 0+1+2+3 per vector lane, then the 8 lanes in
// order) with shuffles, so row means and variances are bit-identical to
// torch.mean on the CPU.
#include "mi_common.cuh"

namespace mi {
namespace rowops {

// Fold one lane's R values in ATen's cascade order (level step 16 for R < 2^16):
// full blocks of 16 rows are summed into level 0 and moved into level 1, the
// remainder goes into level 0, and the result is level0 + level1 (+0 +0 for
// the two unused levels, which only matters for the sign of a zero).
template <int R>
__device__ __forceinline__ float lane_cascade(const float (&v)[R]) {
    float l0 = 0.0f, l1 = 0.0f;
    constexpr int FULL = (R / 16) * 16;
#pragma unroll
    for (int i = 0; i < FULL; i += 16) {
        float c = 0.0f;  // level 0 restarts from 0 after every cascade step
#pragma unroll
        for (int j = 0; j < 16; j++) c = __fadd_rn(c, v[i + j]);
        l1 = __fadd_rn(l1, c);  // acc[1] += acc[0]
    }
#pragma unroll
    for (int i = FULL; i < R; i++) l0 = __fadd_rn(l0, v[i]);
    float a = __fadd_rn(l0, l1);
    a = __fadd_rn(a, 0.0f);
    a = __fadd_rn(a, 0.0f);
    return a;
}

// Combine the 32 lane partials in ATen's order; every lane returns the total.
__device__ __forceinline__ float warp_combine(float p) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    float p8 = __shfl_sync(FULL, p, (lane + 8) & 31);
    float p16 = __shfl_sync(FULL, p, (lane + 16) & 31);
    float p24 = __shfl_sync(FULL, p, (lane + 24) & 31);
    float q = __fadd_rn(__fadd_rn(__fadd_rn(p, p8), p16), p24);  // valid in lanes 0..7
    float tot = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) tot = __fadd_rn(tot, __shfl_sync(FULL, q, j));
    return tot;
}

template <int R>
__device__ __forceinline__ float row_mean(const float (&v)[R]) {
    return __fdiv_rn(warp_combine(lane_cascade<R>(v)), (float)(32 * R));
}

// NaN-propagating warp max of |y| (torch.amax semantics)
__device__ __forceinline__ float warp_absmax(float m, bool nan) {
    const unsigned FULL = 0xffffffffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, o));
    nan = __any_sync(FULL, nan);
    return nan ? __int_as_float(0x7fc00000) : m;
}

// Row pre-pass.  MODE bits: 1 = embedding gather, 2 = residual add,
// 4 = write x_out, 8 = write y_norm, 16 = quantise, 32 = write inv_rms,
// 64 = centre once (BitShiftNormFunction alone) instead of twice.
template <int R>
__global__ void __launch_bounds__(256)
rowprep_kernel(const float* x, const float* delta, const float* __restrict__ res_gate,
               const int64_t* __restrict__ ids, const float* __restrict__ emb, int vocab, float* x_out,
               const float* __restrict__ gamma, const float* __restrict__ step, float* __restrict__ y_norm,
               int8_t* __restrict__ xq, float* __restrict__ xscale, float* __restrict__ inv_rms, int T, int mode) {
    // x / delta / x_out are not __restrict__: the residual stream is updated in
    // place (each lane reads its elements before writing the same elements).
    constexpr int D = 32 * R;
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    grid_dependency_sync();
    const float g = (mode & 2) ? *res_gate : 0.0f;
    const float stp = *step;
    float gam[R];
#pragma unroll
    for (int r = 0; r < R; r++) gam[r] = gamma[32 * r + lane];

    for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
        float v[R];
        const float* src = x + (size_t)t * D;
        bool zero_row = false;
        if (mode & 1) {
            const int64_t id = ids[t];
            zero_row = (id < 0) || (id >= vocab);
            if (zero_row && lane == 0) raise_dev_error(MI_DEV_PRECOND);
            src = emb + (size_t)(zero_row ? 0 : id) * D;
        }
#pragma unroll
        for (int r = 0; r < R; r++) v[r] = zero_row ? 0.0f : src[32 * r + lane];
        if (mode & 2) {
            const float* dl = delta + (size_t)t * D;
#pragma unroll
            for (int r = 0; r < R; r++) v[r] = __fadd_rn(v[r], __fmul_rn(dl[32 * r + lane], g));
        }
        if (mode & 4) {
#pragma unroll
            for (int r = 0; r < R; r++) x_out[(size_t)t * D + 32 * r + lane] = v[r];
        }
        if (!(mode & (8 | 16 | 32))) continue;  // residual update only
        // BitShiftNorm.forward: x - mean(x) (src/mamba_integer_model.py:463);
        // skipped when the caller is BitShiftNormFunction itself (mode 64)
        if (!(mode & 64)) {
            float m1 = row_mean<R>(v);
#pragma unroll
            for (int r = 0; r < R; r++) v[r] = __fsub_rn(v[r], m1);
        }
        // BitShiftNormFunction.forward: centre again, var = mean(xc^2) (:202-205)
        float m2 = row_mean<R>(v);
        float sq[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            v[r] = __fsub_rn(v[r], m2);
            sq[r] = __fmul_rn(v[r], v[r]);
        }
        float var = row_mean<R>(sq);
        float s = pow2_scale(var);
        if ((mode & 32) && lane == 0) inv_rms[t] = s;
        // ((xc * s) * gamma) * step_size (:222)
        float am = 0.0f;
        bool nan = false;
#pragma unroll
        for (int r = 0; r < R; r++) {
            float y = __fmul_rn(__fmul_rn(__fmul_rn(v[r], s), gam[r]), stp);
            v[r] = y;
            float a = fabsf(y);
            nan |= (a != a);
            am = fmaxf(am, a);
        }
        if (mode & 8) {
#pragma unroll
            for (int r = 0; r < R; r++) y_norm[(size_t)t * D + 32 * r + lane] = v[r];
        }
        if (mode & 16) {
            // activation_quant_dynamic (src/rational_bitnet.py:102-111)
            float amax = warp_absmax(am, nan);
            float sc = clamp_t(amax, 1e-8f, __int_as_float(0x7f800000));
            float inv = __fmul_rn(__frcp_rn(sc), 127.0f);  // Tensor.__rdiv__: reciprocal * 127
#pragma unroll
            for (int r = 0; r < R; r++) xq[(size_t)t * D + 32 * r + lane] = (int8_t)quant_i8(__fmul_rn(v[r], inv));
            if (lane == 0) xscale[t] = __fdiv_rn(sc, 127.0f);
        }
    }
}

// Stand-alone per-token quantisation of an arbitrary-width row (two passes:
// absmax, then quantise; the second pass re-reads the row from L1/L2).
__global__ void __launch_bounds__(256)
quant_rows_kernel(const float* __restrict__ x, int ldx, int T, int K, int8_t* __restrict__ xq, int ldq,
                  float* __restrict__ xscale, const float* __restrict__ amax_in, float* __restrict__ clear) {
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    grid_dependency_sync();
    for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
        const float* row = x + (size_t)t * ldx;
        float amax;
        if (amax_in) {
            amax = amax_in[t];  // max |x| of the row, produced by the kernel that wrote x
        } else {
            float am = 0.0f;
            bool nan = false;
            for (int k = lane; k < K; k += 32) {
                float a = fabsf(row[k]);
                nan |= (a != a);
                am = fmaxf(am, a);
            }
            amax = warp_absmax(am, nan);
        }
        float sc = clamp_t(amax, 1e-8f, __int_as_float(0x7f800000));
        float inv = __fmul_rn(__frcp_rn(sc), 127.0f);
        for (int k = lane; k < K; k += 32) xq[(size_t)t * ldq + k] = (int8_t)quant_i8(__fmul_rn(row[k], inv));
        if (lane == 0) {
            xscale[t] = __fdiv_rn(sc, 127.0f);
            if (clear) clear[t] = 0.0f;
        }
    }
}

// quant_rows_kernel for rows of at most 64 values without a given absmax (the
// dt rows of the fused scan): half a warp per row, up to 4 values per lane,
// two rows per warp at once -- the same operations per element, the row's
// absmax and NaN flag reduced over its 16 lanes.
__global__ void __launch_bounds__(256)
quant_rows_narrow_kernel(const float* __restrict__ x, int ldx, int T, int K, int8_t* __restrict__ xq, int ldq,
                         float* __restrict__ xscale, float* __restrict__ clear) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4;
    const int rows_per_cta = (blockDim.x >> 5) * 2;
    grid_dependency_sync();
    for (int t0 = blockIdx.x * rows_per_cta; t0 < T; t0 += gridDim.x * rows_per_cta) {
        const int t = t0 + (threadIdx.x >> 5) * 2 + half;
        const bool okr = t < T;
        float v[4];
        float am = 0.0f;
        bool nan = false;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int k = 4 * hl + e;
            v[e] = (okr && k < K) ? x[(size_t)t * ldx + k] : 0.0f;
            const float a = fabsf(v[e]);
            nan |= (a != a);
            am = fmaxf(am, a);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(FULL, am, o));
        const bool rnan = (__ballot_sync(FULL, nan) >> (16 * half)) & 0xffffu;
        const float amax = rnan ? __int_as_float(0x7fc00000) : am;
        const float sc = clamp_t(amax, 1e-8f, __int_as_float(0x7f800000));
        const float inv = __fmul_rn(__frcp_rn(sc), 127.0f);
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int k = 4 * hl + e;
            if (okr && k < K) xq[(size_t)t * ldq + k] = (int8_t)quant_i8(__fmul_rn(v[e], inv));
        }
        if (okr && hl == 0) {
            xscale[t] = __fdiv_rn(sc, 127.0f);
            if (clear) clear[t] = 0.0f;
        }
    }
}

typedef void (*rowprep_fn)(const float*, const float*, const float*, const int64_t*, const float*, int, float*,
                           const float*, const float*, float*, int8_t*, float*, float*, int, int);

template <int R>
rowprep_fn rowprep_ptr() { return rowprep_kernel<R>; }

static rowprep_fn rowprep_table(int R) {
    switch (R) {
#define MI_R(n) case n: return rowprep_ptr<n>();
        MI_R(1) MI_R(2) MI_R(3) MI_R(4) MI_R(5) MI_R(6) MI_R(7) MI_R(8)
        MI_R(9) MI_R(10) MI_R(11) MI_R(12) MI_R(13) MI_R(14) MI_R(15) MI_R(16)
        MI_R(17) MI_R(18) MI_R(19) MI_R(20) MI_R(21) MI_R(22) MI_R(23) MI_R(24)
        MI_R(25) MI_R(26) MI_R(27) MI_R(28) MI_R(29) MI_R(30) MI_R(31) MI_R(32)
#undef MI_R
        default: return nullptr;
    }
}

static int launch_rowprep(const float* x, const float* delta, const float* res_gate, const int64_t* ids,
                          const float* emb, int vocab, float* x_out, const float* gamma, const float* step, float* y_norm,
                          int8_t* xq, float* xscale, float* inv_rms, int T, int D, int mode, cudaStream_t s) {
    if (T < 0 || D <= 0 || (D % 32) != 0 || D > 1024) return MI_ERR_UNSUPPORTED;
    if (T == 0) return MI_OK;
    rowprep_fn fn = rowprep_table(D / 32);
    if (!fn) return MI_ERR_UNSUPPORTED;
    // one warp per row; few rows (decoding) get 2-warp CTAs so that they spread over
    // more SMs (256 rows: 128 CTAs instead of 32; 1.379 -> 1.368 ms per decode step)
    const int threads = T <= 4096 ? 64 : 256;
    int blocks = cdiv(T, threads / 32);
    if (blocks > 148 * 16) blocks = 148 * 16;
    MI_LAUNCH_DEPENDENT(fn, dim3(blocks), dim3(threads), 0, s, x, delta, res_gate, ids, emb, vocab, x_out, gamma, step,
                        y_norm, xq, xscale, inv_rms, T, mode);
    return MI_OK;
}

}  // namespace rowops
}  // namespace mi

extern "C" int mi_bitshift_norm(const float* x, const float* gamma, const float* step, float* y, float* inv_rms,
                                int T, int D, int center_once, void* stream) {
    if (!x || !gamma || !step || !y) return MI_ERR_INVALID;
    int mode = 8 | (inv_rms ? 32 : 0) | (center_once ? 64 : 0);
    return mi::rowops::launch_rowprep(x, nullptr, nullptr, nullptr, nullptr, 0, nullptr, gamma, step, y, nullptr,
                                      nullptr, inv_rms, T, D, mode, (cudaStream_t)stream);
}

extern "C" int mi_rowprep(const float* x, const float* delta, const float* res_gate, const int64_t* ids,
                          const float* emb, int vocab, float* x_out, const float* gamma, const float* step, float* y_norm,
                          int8_t* xq, float* xscale, int T, int D, void* stream) {
    if (!gamma || !step) return MI_ERR_INVALID;
    int mode = 0;
    if (ids) {
        if (!emb || x || delta || vocab <= 0) return MI_ERR_INVALID;
        mode |= 1;
    } else if (!x) {
        return MI_ERR_INVALID;
    }
    if (delta) {
        if (!res_gate) return MI_ERR_INVALID;
        mode |= 2;
    }
    if (x_out) mode |= 4;
    if (y_norm) mode |= 8;
    if (xq || xscale) {
        if (!xq || !xscale) return MI_ERR_INVALID;
        mode |= 16;
    }
    return mi::rowops::launch_rowprep(x, delta, res_gate, ids, emb, vocab, x_out, gamma, step, y_norm, xq, xscale, nullptr,
                                      T, D, mode, (cudaStream_t)stream);
}

extern "C" int mi_quantize_rows(const float* x, int ldx, int T, int K, int8_t* xq, int ldq, float* xscale,
                                const float* amax, float* clear, void* stream) {
    if (!x || !xq || !xscale) return MI_ERR_INVALID;
    if (T < 0 || K <= 0 || ldx < K || ldq < K) return MI_ERR_INVALID;
    if (T == 0) return MI_OK;
    const int threads = 256;
    if (!amax && K <= 64) {  // narrow rows: two per warp
        int blocks = mi::cdiv(T, threads / 16);
        if (blocks > 148 * 16) blocks = 148 * 16;
        MI_LAUNCH_DEPENDENT(mi::rowops::quant_rows_narrow_kernel, dim3(blocks), dim3(threads), 0, (cudaStream_t)stream,
                            x, ldx, T, K, xq, ldq, xscale, clear);
        return MI_OK;
    }
    int blocks = mi::cdiv(T, threads / 32);
    if (blocks > 148 * 16) blocks = 148 * 16;
    MI_LAUNCH_DEPENDENT(mi::rowops::quant_rows_kernel, dim3(blocks), dim3(threads), 0, (cudaStream_t)stream, x, ldx, T,
                        K, xq, ldq, xscale, amax, clear);
    return MI_OK;
}
