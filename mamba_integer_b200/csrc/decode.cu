// decode.cu -- one generated token for a batch of independent streams:
//   * conv_step_kernel: the causal depthwise conv at the newest position from
//     a per-stream window of the 3 previous conv inputs, ste_clamp +
//     squareplus, int8 quantisation of the row; the window advances;
//   * ssm_step_kernel: int8 quantisation of the step's dt row, the fused
//     dt_proj dot products, decay / dt / u, one convex dyadic update of the
//     16 fp32 states per channel (kept per stream in HBM), y = sum_n h*C, the
//     gate and the int8 quantisation of y;
//   * decode_mid_kernel: the two above with the x_proj BitLinear between them
//     (int8 dot products by dp4a) in one kernel: everything between the
//     in_proj and out_proj GEMMs of a layer;
//   * argmax_rows_kernel: greedy token choice over the logits.
// One CTA per stream: a stream's row never leaves its CTA, so the row absmax
// of each quantisation is a block reduction instead of an atomic.
//
// Every operation is the prefill kernels' own, in the same order, so a token
// decoded here gets the bits MambaIntegerModel.forward gives the last position
// of the full sequence (src/mamba_integer_model.py:396-447, :486-495) -- the
// reference decodes by recomputing that forward for every new token
// (scripts/inference.py:148-160).  The conv keeps the model's order (bias
// first, then one FMA per tap), not the bias-last sum of
// src/cuda_kernels/conv1d_step.cu:30-57.
#include <cooperative_groups.h>

#include "mi_common.cuh"

namespace mi {
namespace decode {

constexpr int STEP_THREADS = 256;
constexpr int MAX_D = 4096;  // channels per stream row
constexpr int CONV_CHUNKS = MAX_D / 4 / STEP_THREADS;   // float4 chunks per thread
constexpr int SSM_CH = MAX_D / STEP_THREADS;            // channels per thread
constexpr int MAX_R16 = 64;                             // dt_rank padded to 16

__device__ __forceinline__ float quant_inv(float amax, float& xscale) { return quant_inv_scale(amax, xscale); }

// Block-wide max of non-negative fp32 bit patterns (NaN sorts above +inf).
__device__ __forceinline__ unsigned block_max_u32(unsigned m, unsigned* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = lane < STEP_THREADS / 32 ? red[lane] : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

// Conv at the newest position for channels c..c+3 of one stream: wrow holds
// the window rows x_{t-3}, x_{t-2}, x_{t-1} (row pitch D), x_t comes from
// xrow; returns squareplus(ste_clamp(conv, +-50)) and advances the window.
__device__ __forceinline__ float4 conv_chunk_step(const float* __restrict__ xrow, float* __restrict__ wrow,
                                                  const float* __restrict__ w, const float* __restrict__ bias, int c,
                                                  int D) {
    const float4 x0 = *reinterpret_cast<const float4*>(wrow + c);
    const float4 x1 = *reinterpret_cast<const float4*>(wrow + D + c);
    const float4 x2 = *reinterpret_cast<const float4*>(wrow + 2 * D + c);
    const float4 x3 = *reinterpret_cast<const float4*>(xrow + c);
    const float4 bs = *reinterpret_cast<const float4*>(bias + c);
    const float xs0[4] = {x0.x, x0.y, x0.z, x0.w}, xs1[4] = {x1.x, x1.y, x1.z, x1.w};
    const float xs2[4] = {x2.x, x2.y, x2.z, x2.w}, xs3[4] = {x3.x, x3.y, x3.z, x3.w};
    const float bv[4] = {bs.x, bs.y, bs.z, bs.w};
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float4 wc = *reinterpret_cast<const float4*>(w + 4 * (c + e));
        // bias first, then one FMA per tap k = 0..3 over positions t-3+k
        float acc = bv[e];
        acc = __fmaf_rn(wc.x, xs0[e], acc);
        acc = __fmaf_rn(wc.y, xs1[e], acc);
        acc = __fmaf_rn(wc.z, xs2[e], acc);
        acc = __fmaf_rn(wc.w, xs3[e], acc);
        r[e] = squareplus_bounded(ste_clamp(acc, -50.0f, 50.0f));
    }
    *reinterpret_cast<float4*>(wrow + c) = x1;
    *reinterpret_cast<float4*>(wrow + D + c) = x2;
    *reinterpret_cast<float4*>(wrow + 2 * D + c) = x3;
    return make_float4(r[0], r[1], r[2], r[3]);
}

__device__ __forceinline__ unsigned absmax_bits4(float4 v) {
    return max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
               max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w))));
}

__device__ __forceinline__ char4 quant4(float4 v, float inv) {
    return make_char4((signed char)quant_i8(__fmul_rn(v.x, inv)), (signed char)quant_i8(__fmul_rn(v.y, inv)),
                      (signed char)quant_i8(__fmul_rn(v.z, inv)), (signed char)quant_i8(__fmul_rn(v.w, inv)));
}

// xz row b: the first D columns are the conv input x_t; win [batch, 3, D]:
// x_{t-3}, x_{t-2}, x_{t-1}.  D % 4 == 0, D <= MAX_D.
__global__ void __launch_bounds__(STEP_THREADS)
conv_step_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ w, const float* __restrict__ bias,
                 float* __restrict__ win, float* __restrict__ act, int8_t* __restrict__ xq,
                 float* __restrict__ xscale, int D) {
    __shared__ unsigned red[STEP_THREADS / 32];
    const int b = blockIdx.x;
    const float* xrow = xz + (size_t)b * ldx;
    float* wrow = win + (size_t)b * 3 * D;
    grid_dependency_sync();
    float4 a[CONV_CHUNKS];
    unsigned m = 0u;
#pragma unroll
    for (int i = 0; i < CONV_CHUNKS; i++) {
        const int c = 4 * (threadIdx.x + i * STEP_THREADS);
        if (c < D) {
            a[i] = conv_chunk_step(xrow, wrow, w, bias, c, D);
            m = max(m, absmax_bits4(a[i]));
            if (act) *reinterpret_cast<float4*>(act + (size_t)b * D + c) = a[i];
        }
    }
    const float amax = __uint_as_float(block_max_u32(m, red));
    float xs;
    const float inv = quant_inv(amax, xs);
#pragma unroll
    for (int i = 0; i < CONV_CHUNKS; i++) {
        const int c = 4 * (threadIdx.x + i * STEP_THREADS);
        if (c < D) *reinterpret_cast<char4*>(xq + (size_t)b * D + c) = quant4(a[i], inv);
    }
    if (threadIdx.x == 0) xscale[b] = xs;
}

// activation_quant_dynamic of the dt row (R values of `row`), as
// mi_quantize_rows computes it, by one full warp: int8 values into dtq (R16
// bytes, zero-padded), the scale into *dts.
__device__ __forceinline__ void dt_row_quant(const float* row, int R, int R16, int32_t* dtq, float* dts) {
    const int lane = threadIdx.x & 31;
    float am = 0.0f;
    bool nan = false;
    for (int k = lane; k < R; k += 32) {
        const float v = fabsf(row[k]);
        nan |= (v != v);
        am = fmaxf(am, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    nan = __any_sync(0xffffffffu, nan);
    const float amax = nan ? __int_as_float(0x7fc00000) : am;
    float xs;
    const float inv = quant_inv(amax, xs);
    int8_t* q8 = reinterpret_cast<int8_t*>(dtq);
    for (int k = lane; k < R16; k += 32) q8[k] = k < R ? (int8_t)quant_i8(__fmul_rn(row[k], inv)) : (int8_t)0;
    if (lane == 0) *dts = xs;
}

// One channel c of the scan step: dt_proj (exact int32 dot product of the
// quantised dt row with w_dt row c, then the BitLinear rescale), decay / dt /
// u, the convex update of its 16 states in hrow (in place), y = sum h*C and
// the gate with zv.  bc = B (16) | C (16).
__device__ __forceinline__ float ssm_channel_step(int c, float actv, float zv, const int32_t* dtq, int R16,
                                                  const int8_t* __restrict__ w_dt, float dscale,
                                                  const float* __restrict__ base, float* hrow, const float* bc) {
    constexpr int NS = 16;
    const int4* wq = reinterpret_cast<const int4*>(w_dt + (size_t)c * R16);
    int acc = 0;
    for (int k = 0; k < R16 / 16; k++) {
        const int4 wv = wq[k];
        acc = __dp4a(dtq[4 * k], wv.x, acc);
        acc = __dp4a(dtq[4 * k + 1], wv.y, acc);
        acc = __dp4a(dtq[4 * k + 2], wv.z, acc);
        acc = __dp4a(dtq[4 * k + 3], wv.w, acc);
    }
    const float mod = ste_clamp(__fmul_rn((float)acc, dscale), -20.0f, 20.0f);                   // (:419-421)
    const float dtv = ste_clamp(__fmul_rn(squareplus_bounded(mod), 0.01f), 0.001f, 0.1f);          // (:425-427)
    const float xdt = __fmul_rn(actv, dtv);
    float4* hp = reinterpret_cast<float4*>(hrow);
    const float4* bp = reinterpret_cast<const float4*>(base + (size_t)c * NS);
    // all 16 states and bases are loaded before the first store: the stores go
    // through the same row pointer, so a load placed after one could not be
    // issued before it, and the four 16-byte pieces would cost four round trips
    float4 hv4[NS / 4], bv4[NS / 4];
#pragma unroll
    for (int q = 0; q < NS / 4; q++) {
        hv4[q] = hp[q];
        bv4[q] = bp[q];
    }
    float yacc = 0.0f;
#pragma unroll
    for (int q = 0; q < NS / 4; q++) {
        float hv[4] = {hv4[q].x, hv4[q].y, hv4[q].z, hv4[q].w};
        const float bv[4] = {bv4[q].x, bv4[q].y, bv4[q].z, bv4[q].w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int n = 4 * q + e;
            // decay_nums = ste_clamp(base + mod, 0, 32000); decay = nums / 2^15   (:423-424, :305)
            const float num = ste_clamp(__fadd_rn(bv[e], mod), 0.0f, 32000.0f);
            const float dec = __fmul_rn(num, 3.0517578125e-05f);
            const float u = __fmul_rn(xdt, bc[n]);
            hv[e] = __fadd_rn(__fmul_rn(hv[e], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));  // (:309)
            yacc = __fmaf_rn(hv[e], bc[NS + n], yacc);                                 // (:440)
        }
        hv4[q] = make_float4(hv[0], hv[1], hv[2], hv[3]);
    }
#pragma unroll
    for (int q = 0; q < NS / 4; q++) hp[q] = hv4[q];
    return sigmoid_gate(yacc, zv);                                                      // (:441-444)
}

// One step of the selective scan for stream b (blockIdx.x).
//   xp row b = [dt (R) | B (16) | C (16)] (the x_proj output, row stride ldxp);
//   act [batch, D]; z rows stride ldz; base [D, 16]; w_dt int8 [D, R16];
//   h [batch, D, 16] fp32 states, updated in place;
//   y (optional) [batch, D]; xq [batch, D] int8 and xscale [batch]: y quantised.
__global__ void __launch_bounds__(STEP_THREADS)
ssm_step_kernel(const float* __restrict__ act, const float* __restrict__ xp, int ldxp, int R,
                const int8_t* __restrict__ w_dt, const float* __restrict__ w_dt_scale, const float* __restrict__ z,
                int ldz, const float* __restrict__ base, float* __restrict__ h, float* __restrict__ y,
                int8_t* __restrict__ xq, float* __restrict__ xscale, int D) {
    constexpr int NS = 16;
    __shared__ __align__(16) int32_t dtq_s[MAX_R16 / 4];
    __shared__ float bc_s[2 * NS];
    __shared__ float dts_s;
    __shared__ unsigned red[STEP_THREADS / 32];
    const int b = blockIdx.x;
    const float* row = xp + (size_t)b * ldxp;
    const int R16 = (R + 15) / 16 * 16;
    grid_dependency_sync();
    if (threadIdx.x < 32) {
        dt_row_quant(row, R, R16, dtq_s, &dts_s);
        bc_s[threadIdx.x] = row[R + threadIdx.x];  // B (16) then C (16)
    }
    __syncthreads();
    const float dscale = __fmul_rn(*w_dt_scale, dts_s);  // (w_scale * x_scale) of the dt_proj BitLinear
    float yv[SSM_CH];
    unsigned m = 0u;
#pragma unroll
    for (int i = 0; i < SSM_CH; i++) {
        const int c = threadIdx.x + i * STEP_THREADS;
        yv[i] = 0.0f;
        if (c >= D) continue;
        yv[i] = ssm_channel_step(c, act[(size_t)b * D + c], z[(size_t)b * ldz + c], dtq_s, R16, w_dt, dscale, base,
                                 h + ((size_t)b * D + c) * NS, bc_s);
        if (y) y[(size_t)b * D + c] = yv[i];
        m = max(m, __float_as_uint(fabsf(yv[i])));
    }
    const float amax = __uint_as_float(block_max_u32(m, red));
    float xs;
    const float inv = quant_inv(amax, xs);
#pragma unroll
    for (int i = 0; i < SSM_CH; i++) {
        const int c = threadIdx.x + i * STEP_THREADS;
        if (c < D) xq[(size_t)b * D + c] = (int8_t)quant_i8(__fmul_rn(yv[i], inv));
    }
    if (threadIdx.x == 0) xscale[b] = xs;
}

// Everything between the in_proj and out_proj GEMMs of one layer for stream
// b: conv step + activation + int8 quantisation (kept in shared memory), the
// x_proj BitLinear as exact int32 dot products (warp w takes outputs w, w+16,
// ...; each lane 16-byte chunks of the row) with the GEMM epilogue's rescale,
// the dt row quantisation, then the scan step and gate (one channel per
// thread per pass, so the 64-byte state rows of a warp are contiguous) and
// the quantisation of y.  w_x int8 [R+32, D];
// xp_out (optional) [batch, R+32] receives the x_proj output.
// D % 16 == 0, D <= MAX_D, R <= 64.
constexpr int MAX_P = MAX_R16 + 32;  // x_proj outputs: dt_rank + 2 * d_state
constexpr int MID_THREADS = 512;     // 16 warps: more state loads in flight per SM
constexpr int MID_CONV = MAX_D / 4 / MID_THREADS;  // conv chunks of 4 channels per thread
constexpr int MID_CH = MAX_D / MID_THREADS;        // scan channels per thread

template <int NT>
__device__ __forceinline__ unsigned block_max_bits(unsigned m, unsigned* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = lane < NT / 32 ? red[lane] : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

__global__ void __launch_bounds__(MID_THREADS, 2)
decode_mid_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ cw, const float* __restrict__ cb,
                  float* __restrict__ win, const int8_t* __restrict__ w_x, const float* __restrict__ w_x_scale,
                  int R, const int8_t* __restrict__ w_dt, const float* __restrict__ w_dt_scale,
                  const float* __restrict__ base, float* __restrict__ h, float* __restrict__ xp_out,
                  int8_t* __restrict__ xq, float* __restrict__ xscale, int D) {
    constexpr int NS = 16;
    constexpr int NW = MID_THREADS / 32;
    constexpr int XCH = MAX_D / 16 / 32;  // 16-byte chunks of the row per lane
    __shared__ __align__(16) float act_s[MAX_D];
    __shared__ __align__(16) int8_t xq_s[MAX_D];
    __shared__ float xp_s[MAX_P];
    __shared__ __align__(16) int32_t dtq_s[MAX_R16 / 4];
    __shared__ float dts_s;
    __shared__ unsigned red[NW];
    __shared__ unsigned red2[NW];
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int P = R + 2 * NS;
    const int R16 = (R + 15) / 16 * 16;
    const float* xrow = xz + (size_t)b * ldx;
    float* wrow = win + (size_t)b * 3 * D;
    grid_dependency_sync();

    // (1) conv + activation on this thread's chunks of 4 channels (into shared memory)
    float4 a[MID_CONV];
    unsigned m = 0u;
#pragma unroll
    for (int i = 0; i < MID_CONV; i++) {
        const int c = 4 * (threadIdx.x + i * MID_THREADS);
        a[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < D) {
            a[i] = conv_chunk_step(xrow, wrow, cw, cb, c, D);
            m = max(m, absmax_bits4(a[i]));
            *reinterpret_cast<float4*>(act_s + c) = a[i];
        }
    }
    // (2) its int8 quantisation, into shared memory
    float xs_c;
    const float inv_c = quant_inv(__uint_as_float(block_max_bits<MID_THREADS>(m, red)), xs_c);
#pragma unroll
    for (int i = 0; i < MID_CONV; i++) {
        const int c = 4 * (threadIdx.x + i * MID_THREADS);
        if (c < D) *reinterpret_cast<char4*>(xq_s + c) = quant4(a[i], inv_c);
    }
    __syncthreads();
    // (3) x_proj: acc * (w_scale * x_scale), as the GEMM epilogue computes it
    const int nch = D / 16;
    const float sc_x = __fmul_rn(*w_x_scale, xs_c);
    for (int o = warp; o < P; o += NW) {
        const int4* wr = reinterpret_cast<const int4*>(w_x + (size_t)o * D);
        int acc = 0;
#pragma unroll
        for (int i = 0; i < XCH; i++) {
            const int j = lane + 32 * i;
            if (j < nch) {
                const int4 wv = wr[j];
                const int4 xv = reinterpret_cast<const int4*>(xq_s)[j];
                acc = __dp4a(xv.x, wv.x, acc);
                acc = __dp4a(xv.y, wv.y, acc);
                acc = __dp4a(xv.z, wv.z, acc);
                acc = __dp4a(xv.w, wv.w, acc);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) {
            const float v = __fmul_rn((float)acc, sc_x);
            xp_s[o] = v;
            if (xp_out) xp_out[(size_t)b * P + o] = v;
        }
    }
    __syncthreads();
    // (4) the dt row's quantisation
    if (warp == 0) dt_row_quant(xp_s, R, R16, dtq_s, &dts_s);
    __syncthreads();
    const float dscale = __fmul_rn(*w_dt_scale, dts_s);
    // (5) scan step + gate, one channel per thread per pass (coalesced state
    // rows); y replaces act in shared memory (same thread, same index);
    // (6) quantisation of y
    unsigned my = 0u;
    for (int i = 0; i < MID_CH; i++) {
        const int c = threadIdx.x + i * MID_THREADS;
        if (c < D) {
            const float yv = ssm_channel_step(c, act_s[c], xrow[D + c], dtq_s, R16, w_dt, dscale, base,
                                              h + ((size_t)b * D + c) * NS, xp_s + R);
            act_s[c] = yv;
            my = max(my, __float_as_uint(fabsf(yv)));
        }
    }
    float xs_y;
    const float inv_y = quant_inv(__uint_as_float(block_max_bits<MID_THREADS>(my, red2)), xs_y);
    for (int i = 0; i < MID_CH; i++) {
        const int c = threadIdx.x + i * MID_THREADS;
        if (c < D) xq[(size_t)b * D + c] = (int8_t)quant_i8(__fmul_rn(act_s[c], inv_y));
    }
    if (threadIdx.x == 0) xscale[b] = xs_y;
}

// decode_mid_kernel split over a cluster of MC_CS CTAs per stream: CTA rank r
// takes channels [r*D/MC_CS, (r+1)*D/MC_CS).  The three row-wide quantities --
// the conv output's absmax, the x_proj dot products (each over all D
// channels) and y's absmax -- are combined through distributed shared
// memory: each CTA leaves its partial (a max, or exact int32 partial dot
// products) in its shared memory, the cluster synchronises, and every CTA
// reads all MC_CS partials.  A max and an integer sum do not depend on the
// order they are combined in, so the results are those of decode_mid_kernel
// bit for bit.  256 streams become 1024 CTAs, which fill the SMs evenly where
// one 512-thread CTA per stream left most SMs with one or two.
// 4 CTAs of 128 threads per stream measured fastest at config 5 (256 streams, d_inner 2048):
// 1.51 ms per decode step, against 1.57 for one 512-thread CTA per stream, 1.57 for 2 x 128,
// 1.62 for 4 x 64, 1.73 for 4 x 256, 1.78 for 8 x 128.
// NT threads a CTA: held to 64 registers, an SM keeps 1024 of them, so the launch
// takes the widest NT (fewest channels a thread walks in series) whose
// batch x 4 x NT threads are still one wave: 128 at 256 streams, 256 at 128, 512 below.
constexpr int MC_CS = 4;          // CTAs per stream (a portable cluster size)
constexpr int MC_XO = 4;          // x_proj outputs per warp pass (int8 weights)
constexpr int MC_XOP = 12;        // x_proj outputs per warp pass (2-bit packed weights)
constexpr int MC_MAX_DC = MAX_D / MC_CS;
constexpr int MC_SM_THREADS = 1024;  // threads an SM keeps at 64 registers

// One channel of the scan step with its 16 states already in registers (hv4,
// updated in place; the caller stores them): dt_proj, decay / dt / u, the
// convex update, y = sum h*C and the gate, in ssm_channel_step's order.
__device__ __forceinline__ float ssm_channel_update(int c, float actv, float zv, const int32_t* dtq, int R16,
                                                    const int8_t* __restrict__ w_dt, float dscale,
                                                    const float* __restrict__ base, float4 (&hv4)[4],
                                                    const float* bc) {
    constexpr int NS = 16;
    const int4* wq = reinterpret_cast<const int4*>(w_dt + (size_t)c * R16);
    const float4* bp = reinterpret_cast<const float4*>(base + (size_t)c * NS);
    // the dt_proj row and the bases are loaded together (R16 <= 64: at most 4 chunks)
    int4 wv[MAX_R16 / 16];
#pragma unroll
    for (int k = 0; k < MAX_R16 / 16; k++) wv[k] = k < R16 / 16 ? wq[k] : make_int4(0, 0, 0, 0);
    float4 bv4[NS / 4];
#pragma unroll
    for (int q = 0; q < NS / 4; q++) bv4[q] = bp[q];
    int acc = 0;
#pragma unroll
    for (int k = 0; k < MAX_R16 / 16; k++) {
        if (k < R16 / 16) {
            acc = __dp4a(dtq[4 * k], wv[k].x, acc);
            acc = __dp4a(dtq[4 * k + 1], wv[k].y, acc);
            acc = __dp4a(dtq[4 * k + 2], wv[k].z, acc);
            acc = __dp4a(dtq[4 * k + 3], wv[k].w, acc);
        }
    }
    const float mod = ste_clamp(__fmul_rn((float)acc, dscale), -20.0f, 20.0f);                   // (:419-421)
    const float dtv = ste_clamp(__fmul_rn(squareplus_bounded(mod), 0.01f), 0.001f, 0.1f);          // (:425-427)
    const float xdt = __fmul_rn(actv, dtv);
    float yacc = 0.0f;
#pragma unroll
    for (int q = 0; q < NS / 4; q++) {
        float hv[4] = {hv4[q].x, hv4[q].y, hv4[q].z, hv4[q].w};
        const float bv[4] = {bv4[q].x, bv4[q].y, bv4[q].z, bv4[q].w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int n = 4 * q + e;
            const float num = ste_clamp(__fadd_rn(bv[e], mod), 0.0f, 32000.0f);                // (:423-424, :305)
            const float dec = __fmul_rn(num, 3.0517578125e-05f);
            const float u = __fmul_rn(xdt, bc[n]);
            hv[e] = __fadd_rn(__fmul_rn(hv[e], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));  // (:309)
            yacc = __fmaf_rn(hv[e], bc[NS + n], yacc);                                 // (:440)
        }
        hv4[q] = make_float4(hv[0], hv[1], hv[2], hv[3]);
    }
    return sigmoid_gate(yacc, zv);                                                      // (:441-444)
}

// PACKED_X: w_x is the 2-bit packed form [R + 2N, D/4] (pack_ternary's layout)
// instead of int8 [R + 2N, D]; a quarter of the bytes for every stream's CTAs
// to read, and each lane loads its weight words for MC_XOP outputs at once.
template <bool PACKED_X, int NT>
__global__ void __cluster_dims__(MC_CS, 1, 1) __launch_bounds__(NT, MC_SM_THREADS / NT)
decode_mid_cluster_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ cw,
                          const float* __restrict__ cb, float* __restrict__ win, const void* __restrict__ w_x_any,
                          const float* __restrict__ w_x_scale, int R, const int8_t* __restrict__ w_dt,
                          const float* __restrict__ w_dt_scale, const float* __restrict__ base,
                          float* __restrict__ h, float* __restrict__ xp_out, int8_t* __restrict__ xq,
                          float* __restrict__ xscale, int D) {
    namespace cg = cooperative_groups;
    constexpr int NS = 16;
    constexpr int NW = NT / 32;
    __shared__ __align__(16) float act_s[MC_MAX_DC];
    __shared__ __align__(16) int8_t xq_s[MC_MAX_DC];
    __shared__ float xp_s[MAX_P];
    __shared__ int part_xp[MAX_P];
    __shared__ __align__(16) int32_t dtq_s[MAX_R16 / 4];
    __shared__ float dts_s;
    __shared__ unsigned red[NW];
    __shared__ unsigned part_amax, part_ymax;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int b = blockIdx.x / MC_CS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int P = R + 2 * NS;
    const int R16 = (R + 15) / 16 * 16;
    const int DC = D / MC_CS;
    const int c0 = rank * DC;
    const float* xrow = xz + (size_t)b * ldx;
    float* wrow = win + (size_t)b * 3 * D;
    float* hbase = h + ((size_t)b * D + c0) * NS;  // this CTA's state rows
    grid_dependency_sync();
    const float wxs = *w_x_scale, wdts = *w_dt_scale;

    // (1) conv + activation of this CTA's channels, into shared memory
    unsigned m = 0u;
    for (int i = threadIdx.x; i < DC / 4; i += NT) {
        const float4 a = conv_chunk_step(xrow, wrow, cw, cb, c0 + 4 * i, D);
        m = max(m, absmax_bits4(a));
        *reinterpret_cast<float4*>(act_s + 4 * i) = a;
    }
    m = block_max_bits<NT>(m, red);
    if (threadIdx.x == 0) part_amax = m;
    cluster.sync();
    // (2) the row's absmax from every CTA's partial, then this CTA's int8 values
    unsigned am = 0u;
#pragma unroll
    for (int r = 0; r < MC_CS; r++) am = max(am, *cluster.map_shared_rank(&part_amax, r));
    float xs_c;
    const float inv_c = quant_inv(__uint_as_float(am), xs_c);
    for (int i = threadIdx.x; i < DC / 4; i += NT)
        *reinterpret_cast<char4*>(xq_s + 4 * i) = quant4(*reinterpret_cast<const float4*>(act_s + 4 * i), inv_c);
    __syncthreads();
    // (3) x_proj: exact int32 partial dot products over this CTA's channels, summed across the
    // cluster.  A warp takes a group of outputs at a time with all their weight loads issued first.
    const int nch = DC / 16;
    if (PACKED_X) {
        // one 32-bit word = 16 ternary weights = one 16-byte chunk of the int8 row
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(w_x_any) + c0 / 16;
        const int wpitch = D / 16;
        for (int o0 = warp * MC_XOP; o0 < P; o0 += NW * MC_XOP) {
            int acc[MC_XOP];
#pragma unroll
            for (int u = 0; u < MC_XOP; u++) acc[u] = 0;
            for (int j = lane; j < nch; j += 32) {
                uint32_t wv[MC_XOP];
#pragma unroll
                for (int u = 0; u < MC_XOP; u++) wv[u] = o0 + u < P ? wp[(size_t)(o0 + u) * wpitch + j] : 0u;
                const int4 xv = reinterpret_cast<const int4*>(xq_s)[j];
#pragma unroll
                for (int u = 0; u < MC_XOP; u++) {
                    const uint4 w16 = mi::gemm::unpack16(wv[u]);
                    acc[u] = __dp4a(xv.x, (int)w16.x, acc[u]);
                    acc[u] = __dp4a(xv.y, (int)w16.y, acc[u]);
                    acc[u] = __dp4a(xv.z, (int)w16.z, acc[u]);
                    acc[u] = __dp4a(xv.w, (int)w16.w, acc[u]);
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
                for (int u = 0; u < MC_XOP; u++) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], off);
            }
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < MC_XOP; u++)
                    if (o0 + u < P) part_xp[o0 + u] = acc[u];
            }
        }
    } else {
        const int8_t* w_x = reinterpret_cast<const int8_t*>(w_x_any);
        for (int o0 = warp * MC_XO; o0 < P; o0 += NW * MC_XO) {
            int acc[MC_XO];
#pragma unroll
            for (int u = 0; u < MC_XO; u++) acc[u] = 0;
            for (int j = lane; j < nch; j += 32) {
                const int4 xv = reinterpret_cast<const int4*>(xq_s)[j];
                int4 wv[MC_XO];
#pragma unroll
                for (int u = 0; u < MC_XO; u++)
                    wv[u] = o0 + u < P ? reinterpret_cast<const int4*>(w_x + (size_t)(o0 + u) * D + c0)[j]
                                       : make_int4(0, 0, 0, 0);
#pragma unroll
                for (int u = 0; u < MC_XO; u++) {
                    acc[u] = __dp4a(xv.x, wv[u].x, acc[u]);
                    acc[u] = __dp4a(xv.y, wv[u].y, acc[u]);
                    acc[u] = __dp4a(xv.z, wv[u].z, acc[u]);
                    acc[u] = __dp4a(xv.w, wv[u].w, acc[u]);
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
                for (int u = 0; u < MC_XO; u++) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], off);
            }
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < MC_XO; u++)
                    if (o0 + u < P) part_xp[o0 + u] = acc[u];
            }
        }
    }
    cluster.sync();
    const float sc_x = __fmul_rn(wxs, xs_c);  // (w_scale * x_scale), as the GEMM epilogue
    for (int o = threadIdx.x; o < P; o += NT) {
        int acc = 0;
#pragma unroll
        for (int r = 0; r < MC_CS; r++) acc += *cluster.map_shared_rank(&part_xp[o], r);
        const float v = __fmul_rn((float)acc, sc_x);
        xp_s[o] = v;
        if (xp_out && rank == 0) xp_out[(size_t)b * P + o] = v;
    }
    __syncthreads();
    // (4) the dt row's quantisation (every CTA of the cluster computes the same)
    if (warp == 0) dt_row_quant(xp_s, R, R16, dtq_s, &dts_s);
    __syncthreads();
    const float dscale = __fmul_rn(wdts, dts_s);
    // (5) scan step + gate of this CTA's channels; y replaces act in shared memory.  (Staging
    // the next channels' states in shared memory by cp.async was slower: the smem it takes
    // comes out of the L1 that holds the weights every stream's CTAs read.)
    unsigned my = 0u;
    for (int i = threadIdx.x; i < DC; i += NT) {
        const int c = c0 + i;
        float4* hp = reinterpret_cast<float4*>(hbase + (size_t)i * NS);
        float4 hv4[NS / 4];
#pragma unroll
        for (int q = 0; q < NS / 4; q++) hv4[q] = hp[q];
        const float yv = ssm_channel_update(c, act_s[i], xrow[D + c], dtq_s, R16, w_dt, dscale, base, hv4, xp_s + R);
#pragma unroll
        for (int q = 0; q < NS / 4; q++) hp[q] = hv4[q];
        act_s[i] = yv;
        my = max(my, __float_as_uint(fabsf(yv)));
    }
    my = block_max_bits<NT>(my, red);
    if (threadIdx.x == 0) part_ymax = my;
    cluster.sync();
    // (6) y's absmax over the cluster, then the int8 values of this CTA's channels
    unsigned ym = 0u;
#pragma unroll
    for (int r = 0; r < MC_CS; r++) ym = max(ym, *cluster.map_shared_rank(&part_ymax, r));
    float xs_y;
    const float inv_y = quant_inv(__uint_as_float(ym), xs_y);
    for (int i = threadIdx.x; i < DC; i += NT)
        xq[(size_t)b * D + c0 + i] = (int8_t)quant_i8(__fmul_rn(act_s[i], inv_y));
    if (threadIdx.x == 0 && rank == 0) xscale[b] = xs_y;
    // No CTA leaves while another may still read its shared memory.  Every remote read
    // (the partial maxima above) has produced its value before its CTA arrives, and
    // nothing is handed over here, so the arrive is relaxed: it does not wait for this
    // CTA's global stores of the row to become visible to the cluster.
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
    asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}

// The cluster kernel at the widest CTA (at most one thread per channel of its
// slice) whose batch x MC_CS CTAs fit the SMs in one wave, with a sixteenth of
// the SMs kept in reserve for the ones a cluster layout leaves idle.
template <bool PACKED_X>
static int launch_mid_cluster(const float* xz, int ldx, const float* conv_w, const float* conv_b, float* win,
                              const void* w_x, const float* w_x_scale, int R, const int8_t* w_dt,
                              const float* w_dt_scale, const float* base, float* h, float* xp_out, int8_t* xq,
                              float* xscale, int batch, int D, cudaStream_t s) {
    const long long room = (long long)mi::gemm::sm_count() * MC_SM_THREADS * 15 / 16;
    const long long ctas = (long long)batch * MC_CS;
    const int DC = D / MC_CS;
    const dim3 grid((unsigned)ctas);
    if (ctas * 512 <= room && DC >= 512) {
        MI_LAUNCH_DEPENDENT(decode_mid_cluster_kernel<PACKED_X, 512>, grid, dim3(512), 0, s, xz, ldx, conv_w, conv_b,
                            win, w_x, w_x_scale, R, w_dt, w_dt_scale, base, h, xp_out, xq, xscale, D);
    } else if (ctas * 256 <= room && DC >= 256) {
        MI_LAUNCH_DEPENDENT(decode_mid_cluster_kernel<PACKED_X, 256>, grid, dim3(256), 0, s, xz, ldx, conv_w, conv_b,
                            win, w_x, w_x_scale, R, w_dt, w_dt_scale, base, h, xp_out, xq, xscale, D);
    } else {
        MI_LAUNCH_DEPENDENT(decode_mid_cluster_kernel<PACKED_X, 128>, grid, dim3(128), 0, s, xz, ldx, conv_w, conv_b,
                            win, w_x, w_x_scale, R, w_dt, w_dt_scale, base, h, xp_out, xq, xscale, D);
    }
    return MI_OK;
}

// torch.argmax over each row: the first index of the maximum, NaN above
// every number (the first NaN wins).
__device__ __forceinline__ bool argmax_better(float v, int i, float bv, int bi) {
    const bool vn = v != v, bn = bv != bv;
    if (vn || bn) return vn && (!bn || i < bi);
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void argmax_take(float v, int i, float& bv, int& bi) {
    if (argmax_better(v, i, bv, bi)) {
        bv = v;
        bi = i;
    }
}

// One CTA of ARGMAX_THREADS per row.  (value, index) pairs are compared by a
// total order, so partial results merge in any order: each thread keeps four
// running maxima (one per float4 component) over 16-byte loads, two loads in
// flight, and the block merges them; rows that are not 16-byte aligned or
// whose width is not a multiple of 4 are scanned element by element.
constexpr int ARGMAX_THREADS = 512;
__global__ void __launch_bounds__(ARGMAX_THREADS)
argmax_rows_kernel(const float* __restrict__ x, int ldx, int V, int64_t* __restrict__ out) {
    __shared__ float sv[ARGMAX_THREADS / 32];
    __shared__ int si[ARGMAX_THREADS / 32];
    const float* row = x + (size_t)blockIdx.x * ldx;
    grid_dependency_sync();
    const float ninf = -__int_as_float(0x7f800000);
    float bv = ninf;
    int bi = 0x7fffffff;
    if (((uintptr_t)row & 15) == 0 && (V & 3) == 0) {
        const float4* row4 = reinterpret_cast<const float4*>(row);
        const int V4 = V >> 2;
        float v0 = ninf, v1 = ninf, v2 = ninf, v3 = ninf;
        int i0 = 0x7fffffff, i1 = 0x7fffffff, i2 = 0x7fffffff, i3 = 0x7fffffff;
        int k = threadIdx.x;
        for (; k + ARGMAX_THREADS < V4; k += 2 * ARGMAX_THREADS) {
            const float4 a = row4[k], c = row4[k + ARGMAX_THREADS];
            argmax_take(a.x, 4 * k, v0, i0);
            argmax_take(a.y, 4 * k + 1, v1, i1);
            argmax_take(a.z, 4 * k + 2, v2, i2);
            argmax_take(a.w, 4 * k + 3, v3, i3);
            const int kc = 4 * (k + ARGMAX_THREADS);
            argmax_take(c.x, kc, v0, i0);
            argmax_take(c.y, kc + 1, v1, i1);
            argmax_take(c.z, kc + 2, v2, i2);
            argmax_take(c.w, kc + 3, v3, i3);
        }
        if (k < V4) {
            const float4 a = row4[k];
            argmax_take(a.x, 4 * k, v0, i0);
            argmax_take(a.y, 4 * k + 1, v1, i1);
            argmax_take(a.z, 4 * k + 2, v2, i2);
            argmax_take(a.w, 4 * k + 3, v3, i3);
        }
        bv = v0;
        bi = i0;
        argmax_take(v1, i1, bv, bi);
        argmax_take(v2, i2, bv, bi);
        argmax_take(v3, i3, bv, bi);
    } else {
        for (int k = threadIdx.x; k < V; k += ARGMAX_THREADS) argmax_take(row[k], k, bv, bi);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        argmax_take(ov, oi, bv, bi);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        bv = lane < ARGMAX_THREADS / 32 ? sv[lane] : ninf;
        bi = lane < ARGMAX_THREADS / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            argmax_take(ov, oi, bv, bi);
        }
        // a row of -inf only: every element ties, index 0
        if (lane == 0) out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

}  // namespace decode
}  // namespace mi

extern "C" int mi_conv_step(const float* xz, int ldx, const float* w, const float* bias, float* win, float* act,
                            int8_t* xq, float* xscale, int batch, int D, void* stream) {
    using namespace mi::decode;
    if (!xz || !w || !bias || !win || !xq || !xscale) return MI_ERR_INVALID;
    if (batch <= 0 || D <= 0 || ldx < D) return MI_ERR_INVALID;
    if (D % 4 != 0 || D > MAX_D || ldx % 4 != 0 || batch > 2147483647 / 4) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)xz | (uintptr_t)w | (uintptr_t)bias | (uintptr_t)win | (uintptr_t)act) & 15) return MI_ERR_INVALID;
    if (((uintptr_t)xq) & 3) return MI_ERR_INVALID;
    MI_LAUNCH_DEPENDENT(conv_step_kernel, dim3(batch), dim3(STEP_THREADS), 0, (cudaStream_t)stream, xz, ldx, w, bias,
                        win, act, xq, xscale, D);
    return MI_OK;
}

extern "C" int mi_ssm_step(const float* act, const float* xp, int ldxp, int R, const int8_t* w_dt,
                           const float* w_dt_scale, const float* z, int ldz, const float* base, float* h, float* y,
                           int8_t* xq, float* xscale, int batch, int D, int N, void* stream) {
    using namespace mi::decode;
    if (!act || !xp || !w_dt || !w_dt_scale || !z || !base || !h || !xq || !xscale) return MI_ERR_INVALID;
    if (N != 16) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || D <= 0 || R <= 0 || ldxp < R + 2 * N || ldz < D) return MI_ERR_INVALID;
    if (D > MAX_D || (R + 15) / 16 * 16 > MAX_R16) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)h | (uintptr_t)base | (uintptr_t)w_dt) & 15) return MI_ERR_INVALID;
    MI_LAUNCH_DEPENDENT(ssm_step_kernel, dim3(batch), dim3(STEP_THREADS), 0, (cudaStream_t)stream, act, xp, ldxp, R,
                        w_dt, w_dt_scale, z, ldz, base, h, y, xq, xscale, D);
    return MI_OK;
}

extern "C" int mi_decode_mid(const float* xz, int ldx, const float* conv_w, const float* conv_b, float* win,
                             const int8_t* w_x, const float* w_x_scale, int R, const int8_t* w_dt,
                             const float* w_dt_scale, const float* base, float* h, float* xp_out, int8_t* xq,
                             float* xscale, int batch, int D, int N, void* stream) {
    using namespace mi::decode;
    if (!xz || !conv_w || !conv_b || !win || !w_x || !w_x_scale || !w_dt || !w_dt_scale || !base || !h || !xq ||
        !xscale)
        return MI_ERR_INVALID;
    if (N != 16) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || D <= 0 || R <= 0 || ldx < 2 * D) return MI_ERR_INVALID;
    if (D % 16 != 0 || D > MAX_D || (R + 15) / 16 * 16 > MAX_R16 || ldx % 4 != 0) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)xz | (uintptr_t)conv_w | (uintptr_t)conv_b | (uintptr_t)win | (uintptr_t)w_x | (uintptr_t)h |
         (uintptr_t)base | (uintptr_t)w_dt) & 15)
        return MI_ERR_INVALID;
    if (((uintptr_t)xq) & 3) return MI_ERR_INVALID;
    if (D % (16 * MC_CS) == 0 && (long long)batch * MC_CS <= 0x7fffffffLL) {
        // a cluster of MC_CS CTAs per stream (each channel slice a multiple of 16 bytes of int8)
        return launch_mid_cluster<false>(xz, ldx, conv_w, conv_b, win, w_x, w_x_scale, R, w_dt, w_dt_scale, base, h,
                                         xp_out, xq, xscale, batch, D, (cudaStream_t)stream);
    } else {
        MI_LAUNCH_DEPENDENT(decode_mid_kernel, dim3(batch), dim3(MID_THREADS), 0, (cudaStream_t)stream, xz, ldx,
                            conv_w, conv_b, win, w_x, w_x_scale, R, w_dt, w_dt_scale, base, h, xp_out, xq, xscale, D);
    }
    return MI_OK;
}

extern "C" int mi_decode_mid_packed(const float* xz, int ldx, const float* conv_w, const float* conv_b, float* win,
                                    const uint8_t* w_x_packed, const float* w_x_scale, int R, const int8_t* w_dt,
                                    const float* w_dt_scale, const float* base, float* h, float* xp_out,
                                    int8_t* xq, float* xscale, int batch, int D, int N, void* stream) {
    using namespace mi::decode;
    if (!xz || !conv_w || !conv_b || !win || !w_x_packed || !w_x_scale || !w_dt || !w_dt_scale || !base || !h ||
        !xq || !xscale)
        return MI_ERR_INVALID;
    if (N != 16) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || D <= 0 || R <= 0 || ldx < 2 * D) return MI_ERR_INVALID;
    // each CTA's channel slice is a whole number of 16-weight words
    if (D % (16 * MC_CS) != 0 || D > MAX_D || (R + 15) / 16 * 16 > MAX_R16 || ldx % 4 != 0)
        return MI_ERR_UNSUPPORTED;
    if ((long long)batch * MC_CS > 0x7fffffffLL) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)xz | (uintptr_t)conv_w | (uintptr_t)conv_b | (uintptr_t)win | (uintptr_t)h | (uintptr_t)base |
         (uintptr_t)w_dt) & 15)
        return MI_ERR_INVALID;
    if (((uintptr_t)w_x_packed | (uintptr_t)xq) & 3) return MI_ERR_INVALID;
    return launch_mid_cluster<true>(xz, ldx, conv_w, conv_b, win, w_x_packed, w_x_scale, R, w_dt, w_dt_scale, base,
                                    h, xp_out, xq, xscale, batch, D, (cudaStream_t)stream);
}

extern "C" int mi_argmax_rows(const float* x, int ldx, int T, int V, int64_t* out, void* stream) {
    using namespace mi::decode;
    if (!x || !out || T <= 0 || V <= 0 || ldx < V) return MI_ERR_INVALID;
    MI_LAUNCH_DEPENDENT(argmax_rows_kernel, dim3(T), dim3(ARGMAX_THREADS), 0, (cudaStream_t)stream, x, ldx, V, out);
    return MI_OK;
}
