// ssm.cu -- the selective-scan half of MambaIntegerBlock on sm_100a:
//   * causal depthwise conv + ste_clamp + squareplus (+ row absmax), one
//     thread per (sequence, channel) walking the positions, then the int8
//     quantisation that feeds x_proj;
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
// One thread per (sequence, 4 adjacent channels) walks a chunk of CONV_TC
// positions with the 4-tap windows in registers, so every input element is
// read once with 16-byte loads, coalesced across channels.  The row absmax
// needed by the following int8 quantisation is accumulated with one
// atomicMax per warp and position into amax (fp32 bits of non-negative
// values order like unsigned integers; NaN sorts above +inf, which makes a
// NaN row propagate as torch.amax does).
constexpr int CONV_THREADS = 128;
constexpr int CONV_TC = 64;  // positions per CTA
constexpr int CONV_G = 8;    // positions per group: computed together, absmax reduced together

__device__ __forceinline__ float conv_tap4(float bs, float4 wc, float x0, float x1, float x2, float x3) {
    // bias first, then one FMA per tap k = 0..3 over positions t-3+k
    float acc = bs;
    acc = __fmaf_rn(wc.x, x0, acc);
    acc = __fmaf_rn(wc.y, x1, acc);
    acc = __fmaf_rn(wc.z, x2, acc);
    acc = __fmaf_rn(wc.w, x3, acc);
    return squareplus_bounded(ste_clamp(acc, -50.0f, 50.0f));
}

// xz: [batch*L, ldx], conv input = columns [0, D).  act: [batch*L, D].  D % 4 == 0.
__global__ void __launch_bounds__(CONV_THREADS)
conv_act_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ w, const float* __restrict__ bias,
                float* __restrict__ act, unsigned int* __restrict__ amax, int L, int D) {
    const int c = 4 * (blockIdx.x * CONV_THREADS + threadIdx.x);  // first of this thread's 4 channels
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.y;
    const int t0 = blockIdx.z * CONV_TC;
    const bool active = c < D;
    const int cc = active ? c : 0;
    float4 wv[4];
#pragma unroll
    for (int e = 0; e < 4; e++) wv[e] = *reinterpret_cast<const float4*>(w + 4 * (cc + e));
    const float4 bs = *reinterpret_cast<const float4*>(bias + cc);
    const size_t row0 = (size_t)b * L;
    const float* px = xz + row0 * ldx + cc;
    const float4 zero4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    // windows x[t-3], x[t-2], x[t-1] of the 4 channels
    float4 w0 = (t0 - 3 >= 0) ? *reinterpret_cast<const float4*>(px + (size_t)(t0 - 3) * ldx) : zero4;
    float4 w1 = (t0 - 2 >= 0) ? *reinterpret_cast<const float4*>(px + (size_t)(t0 - 2) * ldx) : zero4;
    float4 w2 = (t0 - 1 >= 0) ? *reinterpret_cast<const float4*>(px + (size_t)(t0 - 1) * ldx) : zero4;
    const int tend = min(L, t0 + CONV_TC);
    for (int t = t0; t < tend; t += CONV_G) {
        float4 xv[CONV_G];
#pragma unroll
        for (int j = 0; j < CONV_G; j++)
            xv[j] = (t + j < tend) ? __ldg(reinterpret_cast<const float4*>(px + (size_t)(t + j) * ldx)) : zero4;
        unsigned m[CONV_G];
#pragma unroll
        for (int j = 0; j < CONV_G; j++) {
            float4 a;
            a.x = conv_tap4(bs.x, wv[0], w0.x, w1.x, w2.x, xv[j].x);
            a.y = conv_tap4(bs.y, wv[1], w0.y, w1.y, w2.y, xv[j].y);
            a.z = conv_tap4(bs.z, wv[2], w0.z, w1.z, w2.z, xv[j].z);
            a.w = conv_tap4(bs.w, wv[3], w0.w, w1.w, w2.w, xv[j].w);
            w0 = w1;
            w1 = w2;
            w2 = xv[j];
            const bool ok = active && (t + j < tend);
            if (ok) *reinterpret_cast<float4*>(act + (row0 + t + j) * D + c) = a;
            const unsigned mx = max(max(__float_as_uint(fabsf(a.x)), __float_as_uint(fabsf(a.y))),
                                    max(__float_as_uint(fabsf(a.z)), __float_as_uint(fabsf(a.w))));
            m[j] = ok ? mx : 0u;
        }
        // row absmax of the group's positions: butterflies interleaved over the group
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int j = 0; j < CONV_G; j++) m[j] = max(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
        }
        unsigned mine = 0u;  // lane j publishes position t + j
#pragma unroll
        for (int j = 0; j < CONV_G; j++) mine = (lane == j) ? m[j] : mine;
        if (lane < CONV_G && t + lane < tend) atomicMax(amax + row0 + t + lane, mine);
    }
}

// Row-owning variant with the quantisation fused: one CTA holds whole rows
// (all D channels, 4 adjacent channels per thread) for a chunk of CONV_TC
// positions of one sequence, so the absmax of each position's row is a block
// reduction and the int8 quantisation follows from the registers -- no second
// pass over act, no atomics, no workspace.  Same arithmetic as
// conv_act_kernel followed by quant_rows_kernel.
constexpr int CONVR_G = 4;  // positions per group (one block reduction each group)
constexpr int CONVR_RING = 3;  // groups of input rows staged in shared memory

__device__ __forceinline__ void conv_cp16(float* smem, const float* gmem, bool pred) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem), "r"(pred ? 16 : 0)
                 : "memory");
}

// MAXT = the CTA size it is compiled for: up to 384 threads (D <= 1536) it
// gets up to 80 registers at two CTAs per SM and computes the channels in
// f32x2 pairs; up to 1024 threads it stays within 64 registers, scalar.
// The input rows arrive through a ring of CONVR_RING groups in dynamic shared
// memory ([CONVR_RING][CONVR_G][D] floats), two groups ahead of the one being
// computed; each thread copies and reads only its own 16-byte chunks, so the
// ring needs no barrier of its own.
template <int MAXT>
__global__ void __launch_bounds__(MAXT, MAXT <= 384 ? 2 : 1)
conv_rows_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ w, const float* __restrict__ bias,
                 float* __restrict__ act, int8_t* __restrict__ xq, float* __restrict__ xscale, int L, int D) {
    constexpr bool PAIRED = MAXT <= 384;
    __shared__ unsigned red[2][CONVR_G][32];  // per position: each warp's max |act| bits (double buffer)
    extern __shared__ __align__(16) float xring[];
    const int c = 4 * threadIdx.x;  // first of this thread's 4 channels
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int b = blockIdx.y;
    const int t0 = blockIdx.x * CONV_TC;
    const bool active = c < D;
    const int cc = active ? c : 0;
    grid_dependency_sync();
    float4 wv[4];
#pragma unroll
    for (int e = 0; e < 4; e++) wv[e] = *reinterpret_cast<const float4*>(w + 4 * (cc + e));
    const float4 bs = *reinterpret_cast<const float4*>(bias + cc);
    const size_t row0 = (size_t)b * L;
    const float* px = xz + row0 * ldx + cc;
    const float4 zero4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float4 w0 = (t0 - 3 >= 0) ? *reinterpret_cast<const float4*>(px + (size_t)(t0 - 3) * ldx) : zero4;
    float4 w1 = (t0 - 2 >= 0) ? *reinterpret_cast<const float4*>(px + (size_t)(t0 - 2) * ldx) : zero4;
    float4 w2 = (t0 - 1 >= 0) ? *reinterpret_cast<const float4*>(px + (size_t)(t0 - 1) * ldx) : zero4;
    const int tend = min(L, t0 + CONV_TC);
    // rows t .. t + CONVR_G - 1 into ring slot `slot` (rows past tend read as zero)
    auto stage = [&](int t, int slot) {
        if (active) {
#pragma unroll
            for (int j = 0; j < CONVR_G; j++) {
                const bool ok = t + j < tend;
                conv_cp16(xring + (size_t)(slot * CONVR_G + j) * D + c, px + (size_t)(ok ? t + j : t0) * ldx, ok);
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    stage(t0, 0);
    stage(t0 + CONVR_G, 1);
    int buf = 0, slot = 0;
    for (int t = t0; t < tend; t += CONVR_G, buf ^= 1, slot = slot == CONVR_RING - 1 ? 0 : slot + 1) {
        float4 a[CONVR_G];
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");  // this group's rows have landed
#pragma unroll
        for (int j = 0; j < CONVR_G; j++)
            a[j] = active ? *reinterpret_cast<const float4*>(xring + (size_t)(slot * CONVR_G + j) * D + c) : zero4;
        // the group after next goes to the slot read two groups ago
        stage(t + 2 * CONVR_G, slot == 0 ? CONVR_RING - 1 : slot - 1);
        unsigned m[CONVR_G];
#pragma unroll
        for (int j = 0; j < CONVR_G; j++) {
            const float4 xv = a[j];
            if (PAIRED) {
                // channels (x, y) and (z, w) in pairs: the FMA taps (bias first,
                // k = 0..3), ste_clamp and squareplus as f32x2
                float2 p = make_float2(bs.x, bs.y), q = make_float2(bs.z, bs.w);
                p = __ffma2_rn(make_float2(wv[0].x, wv[1].x), make_float2(w0.x, w0.y), p);
                q = __ffma2_rn(make_float2(wv[2].x, wv[3].x), make_float2(w0.z, w0.w), q);
                p = __ffma2_rn(make_float2(wv[0].y, wv[1].y), make_float2(w1.x, w1.y), p);
                q = __ffma2_rn(make_float2(wv[2].y, wv[3].y), make_float2(w1.z, w1.w), q);
                p = __ffma2_rn(make_float2(wv[0].z, wv[1].z), make_float2(w2.x, w2.y), p);
                q = __ffma2_rn(make_float2(wv[2].z, wv[3].z), make_float2(w2.z, w2.w), q);
                p = __ffma2_rn(make_float2(wv[0].w, wv[1].w), make_float2(xv.x, xv.y), p);
                q = __ffma2_rn(make_float2(wv[2].w, wv[3].w), make_float2(xv.z, xv.w), q);
                p = squareplus_bounded2(ste_clamp2(p, -50.0f, 50.0f));
                q = squareplus_bounded2(ste_clamp2(q, -50.0f, 50.0f));
                a[j] = make_float4(p.x, p.y, q.x, q.y);
            } else {
                a[j].x = conv_tap4(bs.x, wv[0], w0.x, w1.x, w2.x, xv.x);
                a[j].y = conv_tap4(bs.y, wv[1], w0.y, w1.y, w2.y, xv.y);
                a[j].z = conv_tap4(bs.z, wv[2], w0.z, w1.z, w2.z, xv.z);
                a[j].w = conv_tap4(bs.w, wv[3], w0.w, w1.w, w2.w, xv.w);
            }
            w0 = w1;
            w1 = w2;
            w2 = xv;
            const bool ok = active && (t + j < tend);
            if (ok) *reinterpret_cast<float4*>(act + (row0 + t + j) * D + c) = a[j];
            const unsigned mx = max(max(__float_as_uint(fabsf(a[j].x)), __float_as_uint(fabsf(a[j].y))),
                                    max(__float_as_uint(fabsf(a[j].z)), __float_as_uint(fabsf(a[j].w))));
            m[j] = ok ? mx : 0u;  // fp32 bits of non-negative values order like unsigned ints, NaN on top
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int j = 0; j < CONVR_G; j++) m[j] = max(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
        }
        if (lane < CONVR_G) {
            unsigned mine = 0u;
#pragma unroll
            for (int j = 0; j < CONVR_G; j++) mine = (lane == j) ? m[j] : mine;
            red[buf][lane][warp] = mine;
        }
        // one barrier per group: every warp then reduces the per-warp maxima
        // itself (lane j for position j); the buffers alternate, so the next
        // group's writes cannot meet this group's reads
        __syncthreads();
        float inv_l = 0.0f;
        if (lane < CONVR_G) {
            unsigned mm = 0u;
            for (int k = 0; k < nwarps; k++) mm = max(mm, red[buf][lane][k]);
            float xs;
            inv_l = quant_inv_scale(__uint_as_float(mm), xs);
            if (warp == 0 && t + lane < tend) xscale[row0 + t + lane] = xs;
        }
#pragma unroll
        for (int j = 0; j < CONVR_G; j++) {
            const float inv = __shfl_sync(0xffffffffu, inv_l, j);
            if (active && t + j < tend) {
                const char4 q = make_char4((signed char)quant_i8(__fmul_rn(a[j].x, inv)),
                                           (signed char)quant_i8(__fmul_rn(a[j].y, inv)),
                                           (signed char)quant_i8(__fmul_rn(a[j].z, inv)),
                                           (signed char)quant_i8(__fmul_rn(a[j].w, inv)));
                *reinterpret_cast<char4*>(xq + (row0 + t + j) * D + c) = q;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// fused selective scan
// ---------------------------------------------------------------------------
constexpr int NS = 16;
constexpr int SCAN_THREADS = 32;  // one warp per CTA: 32 channels of one sequence
constexpr int SC = 8;             // time steps per staged chunk
constexpr int SSTAGES = 2;        // chunks in flight (double buffer)

// Per-warp staging of one chunk: the four per-step inputs of the warp's 32
// channels (act, decay_mod, z) and the step's B|C row, 4 KB.
struct ScanStage {
    float act[SC][32];
    float mod[SC][32];
    float z[SC][32];
    float bc[SC][2 * NS];
    int32_t dtq[SC][16];  // fused dt_proj: int8 dt row (up to 64 values) as words
    float dts[SC];        // fused dt_proj: per-row activation scale
};
constexpr int MAX_RW = 16;  // dt_rank padded to 16 values <= 64

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(gmem), "r"(pred ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool pred) {
    const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(gmem), "r"(pred ? 4 : 0)
                 : "memory");
}

// Fast-path update of two states (see the decay comment in ssm_scan_kernel):
//   dec = min(base/2^15 + mod/2^15, 32000/2^15),  h = h*dec + (1 - dec)*(x*dt*B).
// The sum, 1 - dec (an FMA with -1: one rounding, as the subtraction) and the
// products are f32x2 operations, whose components round exactly as the scalar
// ones.  An f32x2 add of two f32x2 *products* is contracted into an f32x2 FMA
// by the compiler even with -fmad=false (dropping one product's rounding), so
// the two products of the final sum are written as FMAs with a +0 addend:
// fma(a, b, +0) rounds a*b once, like the product, and the compiler leaves
// the following f32x2 add alone (checked bitwise against the scalar form on
// 4M random operands, and by the parity tests).  fma(a, b, +0) differs from
// a*b only for an exact zero product of negative sign (+0 instead of -0), and
// the sum h*dec + (1 - dec)*u can only see that when (1 - dec)*u is -0 too,
// i.e. when B is -0.0: the model's x_proj output never is (an integer
// accumulator times a positive scale), and a caller passing -0.0 in B may get
// +0.0 where the reference keeps a -0.0 state -- the sign of a zero, nothing
// else.
__device__ __forceinline__ void state_pair_fast(float& h0, float& h1, float b0, float b1, float2 ms2, float2 xdt2,
                                                float B0, float B1) {
    float2 dec = __fadd2_rn(make_float2(b0, b1), ms2);
    dec.x = min_nan(dec.x, 0.9765625f);  // 32000 / 2^15
    dec.y = min_nan(dec.y, 0.9765625f);
    const float2 om = __ffma2_rn(dec, make_float2(-1.0f, -1.0f), make_float2(1.0f, 1.0f));
    const float2 u = __fmul2_rn(xdt2, make_float2(B0, B1));
    const float2 pz = make_float2(0.0f, 0.0f);
    const float2 a1 = __ffma2_rn(make_float2(h0, h1), dec, pz);
    const float2 a2 = __ffma2_rn(om, u, pz);
    const float2 hn = __fadd2_rn(a1, a2);
    h0 = hn.x;
    h1 = hn.y;
}

// Inputs of the decay modulation: either the dt_proj output (RW == 0) or the
// quantised dt rows + scales and the dt_proj weights (RW = words per row).
struct DtSource {
    const float* modraw;   // [T, D] (RW == 0)
    const int8_t* dtq;     // [T, ldq] int8 (RW > 0)
    int ldq;
    const float* dts;      // [T]
    const int8_t* w;       // [D, 4*RW] int8 ternary dt_proj weights
    const float* w_scale;  // [1]
};

// Issue the cp.async copies of chunk [t0, t0+SC) into `st` (16-byte copies).
template <int RW, int CHW>
__device__ __forceinline__ void scan_stage_load(ScanStage& st, const float* __restrict__ act, const DtSource& src,
                                                const float* __restrict__ z, const float* __restrict__ bc, int ldbc,
                                                int ldz, size_t row0, int t0, int L, int d0, int D) {
    const int lane = threadIdx.x & 31;
    constexpr int QR = CHW / 4;  // 16-byte chunks per row of the warp's channels
#pragma unroll
    for (int idx = lane; idx < SC * QR; idx += 32) {  // step r, quarter q
        const int r = idx / QR, q = idx % QR;
        const int t = t0 + r;
        const bool okt = t < L;
        const bool ok = okt && (d0 + 4 * q < D);
        const size_t row = row0 + (okt ? t : 0);
        const int c = d0 + (ok ? 4 * q : 0);
        cp_async16(&st.act[r][4 * q], act + row * D + c, ok);
        if (RW == 0) cp_async16(&st.mod[r][4 * q], src.modraw + row * D + c, ok);
        cp_async16(&st.z[r][4 * q], z + row * ldz + c, ok);
    }
#pragma unroll
    for (int idx = lane; idx < SC * 8; idx += 32) {  // B|C rows: 8 chunks each
        const int r = idx >> 3, q = idx & 7;
        const int t = t0 + r;
        const bool okt = t < L;
        const size_t row = row0 + (okt ? t : 0);
        cp_async16(&st.bc[r][4 * q], bc + row * ldbc + 4 * q, okt);
    }
    if (RW > 0) {
        // dt rows: SC rows x (RW/4) chunks of 16 bytes; scales: SC x 4 bytes
        constexpr int RQ = RW > 0 ? RW / 4 : 1;
        for (int idx = lane; idx < SC * RQ; idx += 32) {
            const int r = idx / RQ, q = idx % RQ;
            const int t = t0 + r;
            const bool okt = t < L;
            const size_t row = row0 + (okt ? t : 0);
            cp_async16(&st.dtq[r][4 * q], src.dtq + row * src.ldq + 16 * q, okt);
        }
        if (lane < SC) {
            const int t = t0 + lane;
            cp_async4(&st.dts[lane], src.dts + row0 + (t < L ? t : 0), t < L);
        }
    }
}

// One warp owns 32/S channels of one sequence; the S lanes of a channel each
// carry 16/S of its fp32 states in registers for the whole sequence (S = 1
// when the layer has enough (sequence, channel) pairs to fill the GPU, 2 or 4
// for small per-GPU batches).  Inputs arrive through a per-warp
// double-buffered cp.async ring of SC-step chunks (no block-level barriers).
// Each chunk is processed in three phases so that only the state recurrence
// is serial: (A) decay clamp / dt / x*dt for SC steps, (B) the convex state
// update and h.C per step, (C) gates, stores and the row absmax reductions for
// SC steps at once.  With S > 1 the h.C accumulation keeps its n = 0..15
// order by continuing the fused multiply-add chain lane after lane.
//
// RW > 0 fuses the dt_proj BitLinear: each lane keeps its channel's ternary
// dt_proj weights (4*RW int8) in registers and forms the exact int32 dot
// product with the step's quantised dt row by dp4a, then applies the
// BitLinear rescale acc * (w_scale * dt_scale[t]) exactly as the GEMM
// epilogue does (src/rational_bitnet.py:204-208).
// (21 one-warp CTAs per SM by registers and shared memory: all 3072 CTAs of a
// 64-sequence x 1536-channel layer are resident at once.)
template <int RW, int S>
__global__ void __launch_bounds__(SCAN_THREADS, 21)
ssm_scan_kernel(const float* __restrict__ act, const float* __restrict__ bc, int ldbc, const DtSource src,
                const float* __restrict__ z, int ldz, const float* __restrict__ base, float* __restrict__ y,
                float* __restrict__ amax, float* __restrict__ h_out, int L, int D) {
    constexpr int CHW = 32 / S;   // channels per warp
    constexpr int NSL = NS / S;   // states per lane
    __shared__ __align__(16) ScanStage stage[SSTAGES];
    const int lane = threadIdx.x;
    const int ch = lane / S;      // channel within the warp
    const int sub = lane % S;     // which slice of the 16 states
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CHW;
    const int d = d0 + ch;
    const bool active = d < D;
    const int dd = active ? d : 0;
    const size_t row0 = (size_t)b * L;

    int32_t wd[RW > 0 ? RW : 1];
    float wsc = 0.0f;
    if (RW > 0) {
        const int4* wrow = reinterpret_cast<const int4*>(src.w + (size_t)dd * (4 * RW));
#pragma unroll
        for (int k = 0; k < RW / 4; k++) {
            const int4 v = wrow[k];
            wd[4 * k] = v.x; wd[4 * k + 1] = v.y; wd[4 * k + 2] = v.z; wd[4 * k + 3] = v.w;
        }
        wsc = *src.w_scale;
    }

    // this lane's states and base / 2^15; the fast-path bounds use all 16 bases
    float h[NSL], bsl[NSL];
    float bmin = __int_as_float(0x7f800000), bmax = -__int_as_float(0x7f800000);
    bool bnan = false;
#pragma unroll
    for (int n = 0; n < NS; n++) {
        const float bv = base[(size_t)dd * NS + n];
        bmin = fminf(bmin, bv);
        bmax = fmaxf(bmax, bv);
        bnan |= (bv != bv);
        if (n / NSL == sub) bsl[n % NSL] = __fmul_rn(bv, 3.0517578125e-05f);
    }
#pragma unroll
    for (int i = 0; i < NSL; i++) h[i] = 0.0f;
    // ste_clamp(., -20, 20) returns values within 20 + 16 of 0 (its error is half an
    // ulp of the input, and inputs whose ulp exceeds 32 give exactly 0), so for bases
    // in [37, 63963] the range conditions of the fast path below always hold
    const bool wide_ok = !bnan && (bmin >= 37.0f) && (bmax <= 63963.0f);

    const int nchunks = cdiv(L, SC);
    scan_stage_load<RW, CHW>(stage[0], act, src, z, bc, ldbc, ldz, row0, 0, L, d0, D);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int c = 0; c < nchunks; c++) {
        ScanStage& st = stage[c & 1];
        if (c + 1 < nchunks)
            scan_stage_load<RW, CHW>(stage[(c + 1) & 1], act, src, z, bc, ldbc, ldz, row0, (c + 1) * SC, L, d0, D);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncwarp();
        const int t0 = c * SC;
        const int tn = min(SC, L - t0);
        float modr[SC];
        if (RW > 0) {
            // decay_mod before its clamp = dt_proj(dt): exact int32 dot product of the
            // int8 dt row with the ternary weights, then acc * (w_scale * dt_scale)
#pragma unroll
            for (int j = 0; j < SC; j++) {
                const int4* q4 = reinterpret_cast<const int4*>(&st.dtq[j][0]);
                int acc = 0;
#pragma unroll
                for (int k = 0; k < RW / 4; k++) {
                    const int4 qv = q4[k];
                    acc = __dp4a(qv.x, wd[4 * k], acc);
                    acc = __dp4a(qv.y, wd[4 * k + 1], acc);
                    acc = __dp4a(qv.z, wd[4 * k + 2], acc);
                    acc = __dp4a(qv.w, wd[4 * k + 3], acc);
                }
                modr[j] = __fmul_rn((float)acc, __fmul_rn(wsc, st.dts[j]));
            }
        } else {
#pragma unroll
            for (int j = 0; j < SC; j++) modr[j] = st.mod[j][ch];
        }

        // (A) per (step, channel): decay_mod, dt_val, x*dt   (:419-428)
        unsigned fast_mask = 0;
        float xdtr[SC];
#pragma unroll
        for (int j = 0; j < SC; j++) {
            const float mod = ste_clamp(modr[j], -20.0f, 20.0f);
            const float dtv = ste_clamp(__fmul_rn(squareplus_bounded(mod), 0.01f), 0.001f, 0.1f);
            modr[j] = mod;
            xdtr[j] = __fmul_rn(st.act[j][ch], dtv);  // x * dt_val
            // decay_nums = ste_clamp(v, 0, 32000), v = base + mod, equals the plain
            // clamp(v, 0, 32000) whenever v <= 64000: for v > 32000 the difference
            // 32000 - v is exact (Sterbenz) so v + (32000 - v) = 32000, for v < 0 it
            // gives +0, and inside the range it is the identity.  Rounding is monotone,
            // so the channel's extreme bases decide.  base >= 1 and a mod that is 0 or
            // not tiny keep base/2^15 and mod/2^15 exact (no subnormals), and with
            // base + mod >= 0 for every state the lower bound cannot bind.
            bool inside = (mod == 0.0f || fabsf(mod) >= 1e-30f);  // false for NaN
            if (!wide_ok)
                inside = inside && !bnan && (bmin >= 1.0f) && (__fadd_rn(bmin, mod) >= 0.0f) &&
                         (__fadd_rn(bmax, mod) <= 64000.0f);
            if (__all_sync(0xffffffffu, inside)) fast_mask |= 1u << j;
            if (S == 1) {  // each lane owns its column: write back at once (fewer live registers)
                st.mod[j][ch] = modr[j];
                st.act[j][ch] = xdtr[j];
            }
        }
        if (S > 1) {
            __syncwarp();  // every lane of a channel has read act before one of them rewrites it
            if (sub == 0) {
#pragma unroll
                for (int j = 0; j < SC; j++) {
                    st.mod[j][ch] = modr[j];
                    st.act[j][ch] = xdtr[j];
                }
            }
        }
        __syncwarp();
        // (B) the recurrence, one step at a time.  A full chunk whose steps all
        // take the fast path runs as one branch-free block (the loads of later
        // steps and the h.C chains of earlier ones overlap); otherwise step by step.
        if (S == 1 && tn == SC && fast_mask == (1u << SC) - 1) {
#pragma unroll
            for (int j = 0; j < SC; j++) {
                const float ms = __fmul_rn(st.mod[j][ch], 3.0517578125e-05f);
                const float xdt = st.act[j][ch];
#pragma unroll
                for (int i = 0; i < NSL; i += 2)
                    state_pair_fast(h[i], h[i + 1], bsl[i], bsl[i + 1], make_float2(ms, ms), make_float2(xdt, xdt),
                                    st.bc[j][i], st.bc[j][i + 1]);
                float yacc = 0.0f;
#pragma unroll
                for (int i = 0; i < NSL; i++) yacc = __fmaf_rn(h[i], st.bc[j][NS + i], yacc);
                st.mod[j][ch] = yacc;
            }
        } else
#pragma unroll 1
        for (int j = 0; j < tn; j++) {
            const float mod = st.mod[j][ch];
            const float xdt = st.act[j][ch];
            const float* Bv = &st.bc[j][sub * NSL];
            const float* Cv = &st.bc[j][NS + sub * NSL];
            if (fast_mask & (1u << j)) {
                // decay = clamp(base + mod, 0, 32000) / 2^15
                //       = min(base/2^15 + mod/2^15, 32000/2^15): both scalings are
                // exact, the sum rounds once, and scaling by 2^-15 commutes with
                // rounding and with the clamp away from subnormals
                const float ms = __fmul_rn(mod, 3.0517578125e-05f);
                // h = h * decay + (1 - decay) * u                       (:309)
#pragma unroll
                for (int i = 0; i < NSL; i += 2)
                    state_pair_fast(h[i], h[i + 1], bsl[i], bsl[i + 1], make_float2(ms, ms), make_float2(xdt, xdt),
                                    Bv[i], Bv[i + 1]);
            } else {
#pragma unroll
                for (int i = 0; i < NSL; i++) {
                    const float bn = __fmul_rn(bsl[i], 32768.0f);  // exact: back to base
                    const float num = ste_clamp(__fadd_rn(bn, mod), 0.0f, 32000.0f);
                    const float dec = __fmul_rn(num, 3.0517578125e-05f);
                    const float u = __fmul_rn(xdt, Bv[i]);
                    h[i] = __fadd_rn(__fmul_rn(h[i], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                }
            }
            // y = matmul(h, C[..., None]): fused multiply-add over n = 0..15 from 0   (:440);
            // the chain passes from the lane holding states [s*NSL, ...) to the next
            float yacc = 0.0f;
#pragma unroll
            for (int s = 0; s < S; s++) {
                const float yin = (s == 0) ? 0.0f : __shfl_up_sync(0xffffffffu, yacc, 1);
                if (sub == s) {
                    yacc = yin;
#pragma unroll
                    for (int i = 0; i < NSL; i++) yacc = __fmaf_rn(h[i], Cv[i], yacc);
                }
            }
            __syncwarp();
            if (sub == S - 1) st.mod[j][ch] = yacc;  // decay_mod of step j is no longer needed
        }
        __syncwarp();
        // (C) gate, store, row absmax                                 (:441-444)
        const bool owner = active && (sub == S - 1);
        unsigned m[SC];
#pragma unroll
        for (int j = 0; j < SC; j++) {
            const float out = sigmoid_gate(st.mod[j][ch], st.z[j][ch]);
            if (j < tn && owner) y[(row0 + t0 + j) * D + d] = out;
            m[j] = (j < tn && owner) ? __float_as_uint(fabsf(out)) : 0u;
        }
        if (amax) {
            // fp32 bits of non-negative values order like unsigned ints (NaN above +inf).
            // Reduce-scatter over the warp: at offsets 16, 8, 4 each lane keeps half
            // of its steps and takes the other half's partner values (9 shuffles for
            // the 8 steps instead of 40); lane 4s + ... ends with step
            // 4*bit4 + 2*bit3 + bit2 of its index.
            static_assert(SC == 8, "reduce-scatter below is written for 8 steps");
            const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
            unsigned m2[4], m3[2];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const unsigned send = b4 ? m[i] : m[4 + i], keep = b4 ? m[4 + i] : m[i];
                m2[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, 16));
            }
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const unsigned send = b3 ? m2[i] : m2[2 + i], keep = b3 ? m2[2 + i] : m2[i];
                m3[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, 8));
            }
            unsigned m4;
            {
                const unsigned send = b2 ? m3[0] : m3[1], keep = b2 ? m3[1] : m3[0];
                m4 = max(keep, __shfl_xor_sync(0xffffffffu, send, 4));
            }
            m4 = max(m4, __shfl_xor_sync(0xffffffffu, m4, 2));
            m4 = max(m4, __shfl_xor_sync(0xffffffffu, m4, 1));
            const int jstep = (b4 ? 4 : 0) + (b3 ? 2 : 0) + (b2 ? 1 : 0);
            if ((lane & 3) == 0 && jstep < tn)
                atomicMax(reinterpret_cast<unsigned int*>(amax) + row0 + t0 + jstep, m4);
        }
        __syncwarp();  // the buffer is refilled by the next iteration's copies
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    if (h_out && active) {
        // final states of the sequence [batch, D, 16] (the decode steps continue from them)
        float* dst = h_out + ((size_t)b * D + d) * NS + sub * NSL;
#pragma unroll
        for (int i = 0; i < NSL; i++) dst[i] = h[i];
    }
}

// Pipelined kernel for small per-GPU batches (few warps per SM, where the
// one-warp kernels above spend most of each chunk waiting on their own
// phases in series).  One CTA owns 32 channels of one sequence, one lane per
// channel as in ssm_scan_kernel<RW, 1>, and splits each chunk's work over
// four warps that work on different chunks at once:
//   warps 0 and 1 stage rows 0-3 / 4-7 of chunk c + PIPE_LA by cp.async and
//          run phase A (decay_mod, dt, x*dt, fast-path vote) of those rows
//          of chunk c;
//   warp 2 runs the recurrence and the h.C contraction of chunk c - 1;
//   warp 3 gates, stores and reduces the row absmax of chunk c - 2.
// Chunks pass through a ring of PIPE_NR staging slots; each slot has three
// named barriers: phase A done (both staging warps arrive, the recurrence
// warp waits), recurrence done (recurrence warp -> gate warp) and gate done
// (gate warp arrives, both staging warps wait before restaging the slot).
// Every warp takes every chunk in order, so each arrival has exactly one
// matching wait (the gate warp signals a slot only when it will be
// restaged), and a warp reaches a slot's barrier for chunk c + NR only after
// the other warps have passed it for chunk c.  The arithmetic is that of
// ssm_scan_kernel<RW, 1>.
constexpr int PIPE_NR = 4;  // ring slots (3 barriers each: 12 ids keep 5 CTAs per SM possible)
constexpr int PIPE_LA = 1;  // chunks staged ahead of the one in phase A
// Sizing, not safety: the gate-done barrier alone keeps restaging safe at any
// staging distance (tests/test_pipe_protocol.py models the hand-offs); with
// PIPE_LA <= PIPE_NR - 3 the staging warps need not wait for a chunk the gate
// warp is still working on.
static_assert(PIPE_LA <= PIPE_NR - 3, "ring sized for a slot in each phase plus the staged ones");
static_assert(3 * PIPE_NR <= 16, "named barrier ids");

// Named barrier `id` in [I, N) issued with its id as an immediate (a run-time
// id makes the compiler reserve all 16 hardware barriers of the CTA, which
// caps the CTAs per SM; immediates reserve only ids below N).
template <int I, int N>
struct NamedBar {
    __device__ __forceinline__ static void arrive(int id, int n) {
        if (id == I) asm volatile("bar.arrive %0, %1;" ::"n"(I), "r"(n) : "memory");
        else NamedBar<I + 1, N>::arrive(id, n);
    }
    __device__ __forceinline__ static void sync(int id, int n) {
        if (id == I) asm volatile("bar.sync %0, %1;" ::"n"(I), "r"(n) : "memory");
        else NamedBar<I + 1, N>::sync(id, n);
    }
};
template <int N>
struct NamedBar<N, N> {
    __device__ __forceinline__ static void arrive(int, int) {}
    __device__ __forceinline__ static void sync(int, int) {}
};

// Stage rows 4*hf .. 4*hf+3 of chunk [t0, t0+SC) (32 channels) into `st`.
template <int RW>
__device__ __forceinline__ void stage_half(ScanStage& st, const float* __restrict__ act, const DtSource& src,
                                           const float* __restrict__ z, const float* __restrict__ bc, int ldbc,
                                           int ldz, size_t row0, int t0, int L, int d0, int D, int hf) {
    const int lane = threadIdx.x & 31;
    {   // act / z (/ mod): 4 rows x 8 chunks of 16 bytes
        const int r = 4 * hf + (lane >> 3), q = lane & 7;
        const int t = t0 + r;
        const bool okt = t < L;
        const bool ok = okt && (d0 + 4 * q < D);
        const size_t row = row0 + (okt ? t : 0);
        const int c = d0 + (ok ? 4 * q : 0);
        cp_async16(&st.act[r][4 * q], act + row * D + c, ok);
        if (RW == 0) cp_async16(&st.mod[r][4 * q], src.modraw + row * D + c, ok);
        cp_async16(&st.z[r][4 * q], z + row * ldz + c, ok);
    }
    {   // B|C: 4 rows x 8 chunks
        const int r = 4 * hf + (lane >> 3), q = lane & 7;
        const int t = t0 + r;
        const bool okt = t < L;
        const size_t row = row0 + (okt ? t : 0);
        cp_async16(&st.bc[r][4 * q], bc + row * ldbc + 4 * q, okt);
    }
    if (RW > 0) {
        constexpr int RQ = RW > 0 ? RW / 4 : 1;
        if (lane < 4 * RQ) {
            const int r = 4 * hf + lane / RQ, q = lane % RQ;
            const int t = t0 + r;
            const bool okt = t < L;
            const size_t row = row0 + (okt ? t : 0);
            cp_async16(&st.dtq[r][4 * q], src.dtq + row * src.ldq + 16 * q, okt);
        }
        if (lane < 4) {
            const int r = 4 * hf + lane;
            const int t = t0 + r;
            cp_async4(&st.dts[r], src.dts + row0 + (t < L ? t : 0), t < L);
        }
    }
}

template <int RW>
__global__ void __launch_bounds__(128)
ssm_scan_pipe_kernel(const float* __restrict__ act, const float* __restrict__ bc, int ldbc, const DtSource src,
                    const float* __restrict__ z, int ldz, const float* __restrict__ base, float* __restrict__ y,
                    float* __restrict__ amax, float* __restrict__ h_out, int L, int D) {
    __shared__ __align__(16) ScanStage ring[PIPE_NR];
    __shared__ unsigned fmask2[PIPE_NR][2];
    // Fixed roles per warp index: the SM already places warp w of its k-th
    // resident CTA on sub-partition (w + k) % 4 (measured), so the recurrence
    // warps of co-resident CTAs land on different sub-partitions.
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * 32;
    const int d = d0 + lane;
    const bool active = d < D;
    const int dd = active ? d : 0;
    const size_t row0 = (size_t)b * L;
    const int nchunks = cdiv(L, SC);
    constexpr int BA = 0, BB = PIPE_NR, BG = 2 * PIPE_NR;  // barrier id bases (no __syncthreads here)
    using Bar = NamedBar<0, 3 * PIPE_NR>;
    if (warp == 2) {
        // ---- recurrence and h.C (ssm_scan_kernel<RW, 1>, phase B)
        float h[NS], bsl[NS];
#pragma unroll
        for (int n = 0; n < NS; n++) {
            bsl[n] = __fmul_rn(base[(size_t)dd * NS + n], 3.0517578125e-05f);
            h[n] = 0.0f;
        }
        for (int c = 0; c < nchunks; c++) {
            const int s = c % PIPE_NR;
            Bar::sync(BA + s, 96);
            ScanStage& st = ring[s];
            const unsigned fm = fmask2[s][0] | fmask2[s][1];
            const int tn = min(SC, L - c * SC);
            if (tn == SC && fm == (1u << SC) - 1) {
#pragma unroll
                for (int j = 0; j < SC; j++) {
                    const float ms = __fmul_rn(st.mod[j][lane], 3.0517578125e-05f);
                    const float xdt = st.act[j][lane];
#pragma unroll
                    for (int i = 0; i < NS; i += 2)
                        state_pair_fast(h[i], h[i + 1], bsl[i], bsl[i + 1], make_float2(ms, ms),
                                        make_float2(xdt, xdt), st.bc[j][i], st.bc[j][i + 1]);
                    float yacc = 0.0f;
#pragma unroll
                    for (int i = 0; i < NS; i++) yacc = __fmaf_rn(h[i], st.bc[j][NS + i], yacc);
                    st.mod[j][lane] = yacc;
                }
            } else {
#pragma unroll 1
                for (int j = 0; j < tn; j++) {
                    const float mod = st.mod[j][lane];
                    const float xdt = st.act[j][lane];
                    if (fm & (1u << j)) {
                        const float ms = __fmul_rn(mod, 3.0517578125e-05f);
#pragma unroll
                        for (int i = 0; i < NS; i += 2)
                            state_pair_fast(h[i], h[i + 1], bsl[i], bsl[i + 1], make_float2(ms, ms),
                                            make_float2(xdt, xdt), st.bc[j][i], st.bc[j][i + 1]);
                    } else {
#pragma unroll
                        for (int i = 0; i < NS; i++) {
                            const float bn = __fmul_rn(bsl[i], 32768.0f);
                            const float num = ste_clamp(__fadd_rn(bn, mod), 0.0f, 32000.0f);
                            const float dec = __fmul_rn(num, 3.0517578125e-05f);
                            const float u = __fmul_rn(xdt, st.bc[j][i]);
                            h[i] = __fadd_rn(__fmul_rn(h[i], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                        }
                    }
                    float yacc = 0.0f;
#pragma unroll
                    for (int i = 0; i < NS; i++) yacc = __fmaf_rn(h[i], st.bc[j][NS + i], yacc);
                    st.mod[j][lane] = yacc;
                }
            }
            __syncwarp();
            Bar::arrive(BB + s, 64);
        }
        if (h_out && active) {
            float* dst = h_out + ((size_t)b * D + d) * NS;
#pragma unroll
            for (int i = 0; i < NS; i++) dst[i] = h[i];
        }
        return;
    }
    if (warp == 3) {
        // ---- gate, store, row absmax (ssm_scan_kernel<RW, 1>, phase C)
        for (int c = 0; c < nchunks; c++) {
            const int s = c % PIPE_NR;
            Bar::sync(BB + s, 64);
            ScanStage& st = ring[s];
            const int t0 = c * SC;
            const int tn = min(SC, L - t0);
            unsigned m[SC];
#pragma unroll
            for (int j = 0; j < SC; j++) {
                const float out = sigmoid_gate(st.mod[j][lane], st.z[j][lane]);
                if (j < tn && active) y[(row0 + t0 + j) * D + d] = out;
                m[j] = (j < tn && active) ? __float_as_uint(fabsf(out)) : 0u;
            }
            __syncwarp();
            if (c < nchunks - PIPE_NR) Bar::arrive(BG + s, 96);  // the slot is restaged with chunk c + NR
            if (amax) {
                const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
                unsigned m2[4], m3[2];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const unsigned send = b4 ? m[i] : m[4 + i], keep = b4 ? m[4 + i] : m[i];
                    m2[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, 16));
                }
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const unsigned send = b3 ? m2[i] : m2[2 + i], keep = b3 ? m2[2 + i] : m2[i];
                    m3[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, 8));
                }
                unsigned m4;
                {
                    const unsigned send = b2 ? m3[0] : m3[1], keep = b2 ? m3[1] : m3[0];
                    m4 = max(keep, __shfl_xor_sync(0xffffffffu, send, 4));
                }
                m4 = max(m4, __shfl_xor_sync(0xffffffffu, m4, 2));
                m4 = max(m4, __shfl_xor_sync(0xffffffffu, m4, 1));
                const int jstep = (b4 ? 4 : 0) + (b3 ? 2 : 0) + (b2 ? 1 : 0);
                if ((lane & 3) == 0 && jstep < tn)
                    atomicMax(reinterpret_cast<unsigned int*>(amax) + row0 + t0 + jstep, m4);
            }
        }
        return;
    }
    // ---- warps 0 and 1: staging and phase A of steps 4*hf .. 4*hf+3 (ssm_scan_kernel<RW, 1>, phase A)
    const int hf = warp;
    int32_t wd[RW > 0 ? RW : 1];
    float wsc = 0.0f;
    if (RW > 0) {
        const int4* wrow = reinterpret_cast<const int4*>(src.w + (size_t)dd * (4 * RW));
#pragma unroll
        for (int k = 0; k < RW / 4; k++) {
            const int4 v = wrow[k];
            wd[4 * k] = v.x; wd[4 * k + 1] = v.y; wd[4 * k + 2] = v.z; wd[4 * k + 3] = v.w;
        }
        wsc = *src.w_scale;
    }
    float bmin = __int_as_float(0x7f800000), bmax = -__int_as_float(0x7f800000);
    bool bnan = false;
#pragma unroll
    for (int n = 0; n < NS; n++) {
        const float bv = base[(size_t)dd * NS + n];
        bmin = fminf(bmin, bv);
        bmax = fmaxf(bmax, bv);
        bnan |= (bv != bv);
    }
    const bool wide_ok = !bnan && (bmin >= 37.0f) && (bmax <= 63963.0f);  // see ssm_scan_kernel
#pragma unroll
    for (int c = 0; c < PIPE_LA; c++) {
        if (c < nchunks) stage_half<RW>(ring[c], act, src, z, bc, ldbc, ldz, row0, c * SC, L, d0, D, hf);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    for (int c = 0; c < nchunks; c++) {
        const int cn = c + PIPE_LA;
        if (cn < nchunks) {
            const int sn = cn % PIPE_NR;
            if (cn >= PIPE_NR) Bar::sync(BG + sn, 96);  // the gate warp is done with chunk cn - NR
            stage_half<RW>(ring[sn], act, src, z, bc, ldbc, ldz, row0, cn * SC, L, d0, D, hf);
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group %0;\n" ::"n"(PIPE_LA) : "memory");
        __syncwarp();
        const int s = c % PIPE_NR;
        ScanStage& st = ring[s];
        unsigned fast_mask = 0;
        // the four rows' decay modulations first, then their squareplus in two
        // f32x2 pairs (squareplus_bounded2: the same roundings per element)
        float modv[4], sqv[4];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int j = 4 * hf + jj;
            float mr;
            if (RW > 0) {
                const int4* q4 = reinterpret_cast<const int4*>(&st.dtq[j][0]);
                int acc0 = 0, acc1 = 0;  // exact: integer sums in any order
#pragma unroll
                for (int k = 0; k < RW / 4; k++) {
                    const int4 qv = q4[k];
                    acc0 = __dp4a(qv.x, wd[4 * k], acc0);
                    acc1 = __dp4a(qv.y, wd[4 * k + 1], acc1);
                    acc0 = __dp4a(qv.z, wd[4 * k + 2], acc0);
                    acc1 = __dp4a(qv.w, wd[4 * k + 3], acc1);
                }
                mr = __fmul_rn((float)(acc0 + acc1), __fmul_rn(wsc, st.dts[j]));
            } else {
                mr = st.mod[j][lane];
            }
            modv[jj] = ste_clamp(mr, -20.0f, 20.0f);
        }
#pragma unroll
        for (int p = 0; p < 2; p++) {
            const float2 sp = squareplus_bounded2(make_float2(modv[2 * p], modv[2 * p + 1]));
            sqv[2 * p] = sp.x;
            sqv[2 * p + 1] = sp.y;
        }
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int j = 4 * hf + jj;
            const float mod = modv[jj];
            const float dtv = ste_clamp(__fmul_rn(sqv[jj], 0.01f), 0.001f, 0.1f);
            bool inside = (mod == 0.0f || fabsf(mod) >= 1e-30f);
            if (!wide_ok)
                inside = inside && !bnan && (bmin >= 1.0f) && (__fadd_rn(bmin, mod) >= 0.0f) &&
                         (__fadd_rn(bmax, mod) <= 64000.0f);
            if (__all_sync(0xffffffffu, inside)) fast_mask |= 1u << j;
            st.mod[j][lane] = mod;
            st.act[j][lane] = __fmul_rn(st.act[j][lane], dtv);  // x * dt_val
        }
        if (lane == 0) fmask2[s][hf] = fast_mask;
        __syncwarp();
        Bar::arrive(BA + s, 96);
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
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

// Split-lane variant (S = 2 or 4 lanes per channel) for small per-GPU batches.
// The S lanes of a channel share its work instead of repeating it:
//   (A) the decay_mod / dt / x*dt prologue of step j is computed by lane
//       j % S of the channel only (the fast-path vote becomes a ballot);
//   (B1) each lane advances its 16/S states for every step and writes the
//       state snapshot of each step to shared memory;
//   (B2) the h.C contractions of the chunk (SC steps x 32/S channels) are
//       spread over the warp, each a 16-term fused multiply-add chain in the
//       reference order n = 0..15 read from the snapshots, so no shuffle sits
//       on the per-step critical path;
//   (C) the gate, store and row absmax of step j again by lane j % S.
template <int RW, int S>
__global__ void __launch_bounds__(SCAN_THREADS)
ssm_scan_split_kernel(const float* __restrict__ act, const float* __restrict__ bc, int ldbc, const DtSource src,
                      const float* __restrict__ z, int ldz, const float* __restrict__ base, float* __restrict__ y,
                      float* __restrict__ amax, float* __restrict__ h_out, int L, int D) {
    static_assert(S == 2 || S == 4 || S == 8, "split variant");
    constexpr int CHW = 32 / S;   // channels per warp
    constexpr int NSL = NS / S;   // states per lane
    constexpr int SPL = SC / S;   // prologue / gate steps per lane
    __shared__ __align__(16) ScanStage stage[SSTAGES];
    __shared__ __align__(16) float snap[SC][32][NSL];
    const int lane = threadIdx.x;
    const int ch = lane / S;
    const int sub = lane % S;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CHW;
    const int d = d0 + ch;
    const bool active = d < D;
    const int dd = active ? d : 0;
    const size_t row0 = (size_t)b * L;
    // lanes with the same sub-index: (lane % S == s) <=> bit pattern
    constexpr unsigned SUBMASK0 = S == 2 ? 0x55555555u : S == 4 ? 0x11111111u : 0x01010101u;

    int32_t wd[RW > 0 ? RW : 1];
    float wsc = 0.0f;
    if (RW > 0) {
        const int4* wrow = reinterpret_cast<const int4*>(src.w + (size_t)dd * (4 * RW));
#pragma unroll
        for (int k = 0; k < RW / 4; k++) {
            const int4 v = wrow[k];
            wd[4 * k] = v.x; wd[4 * k + 1] = v.y; wd[4 * k + 2] = v.z; wd[4 * k + 3] = v.w;
        }
        wsc = *src.w_scale;
    }
    float h[NSL], bsl[NSL];
    float bmin = __int_as_float(0x7f800000), bmax = -__int_as_float(0x7f800000);
    bool bnan = false;
#pragma unroll
    for (int n = 0; n < NS; n++) {
        const float bv = base[(size_t)dd * NS + n];
        bmin = fminf(bmin, bv);
        bmax = fmaxf(bmax, bv);
        bnan |= (bv != bv);
        if (n / NSL == sub) bsl[n % NSL] = __fmul_rn(bv, 3.0517578125e-05f);
    }
#pragma unroll
    for (int i = 0; i < NSL; i++) h[i] = 0.0f;

    const int nchunks = cdiv(L, SC);
    scan_stage_load<RW, CHW>(stage[0], act, src, z, bc, ldbc, ldz, row0, 0, L, d0, D);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int c = 0; c < nchunks; c++) {
        ScanStage& st = stage[c & 1];
        if (c + 1 < nchunks)
            scan_stage_load<RW, CHW>(stage[(c + 1) & 1], act, src, z, bc, ldbc, ldz, row0, (c + 1) * SC, L, d0, D);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncwarp();
        const int t0 = c * SC;
        const int tn = min(SC, L - t0);

        // (A) prologue of steps j = sub, sub + S, ... of this lane's channel   (:419-428)
        unsigned fast_mask = 0;
#pragma unroll
        for (int k = 0; k < SPL; k++) {
            const int j = sub + k * S;
            float mr;
            if (RW > 0) {
                const int4* q4 = reinterpret_cast<const int4*>(&st.dtq[j][0]);
                int acc = 0;
#pragma unroll
                for (int w4 = 0; w4 < RW / 4; w4++) {
                    const int4 qv = q4[w4];
                    acc = __dp4a(qv.x, wd[4 * w4], acc);
                    acc = __dp4a(qv.y, wd[4 * w4 + 1], acc);
                    acc = __dp4a(qv.z, wd[4 * w4 + 2], acc);
                    acc = __dp4a(qv.w, wd[4 * w4 + 3], acc);
                }
                mr = __fmul_rn((float)acc, __fmul_rn(wsc, st.dts[j]));
            } else {
                mr = st.mod[j][ch];
            }
            const float mod = ste_clamp(mr, -20.0f, 20.0f);
            const float dtv = ste_clamp(__fmul_rn(squareplus_bounded(mod), 0.01f), 0.001f, 0.1f);
            st.act[j][ch] = __fmul_rn(st.act[j][ch], dtv);  // x * dt_val (this lane owns (j, ch))
            st.mod[j][ch] = mod;
            // same fast-path condition as the one-lane kernel (see there)
            const bool inside = !active || (!bnan && (bmin >= 1.0f) && (__fadd_rn(bmin, mod) >= 0.0f) &&
                                            (__fadd_rn(bmax, mod) <= 64000.0f) &&
                                            (mod == 0.0f || fabsf(mod) >= 1e-30f));
            const unsigned bal = __ballot_sync(0xffffffffu, inside);
#pragma unroll
            for (int s = 0; s < S; s++) {
                const unsigned m = SUBMASK0 << s;
                if ((bal & m) == m) fast_mask |= 1u << (s + k * S);
            }
        }
        __syncwarp();
        // (B1) state recurrence; snapshot of every step (a full all-fast chunk as
        // one branch-free block, as in the one-lane kernel)
        if (tn == SC && fast_mask == (1u << SC) - 1) {
#pragma unroll
            for (int j = 0; j < SC; j++) {
                const float ms = __fmul_rn(st.mod[j][ch], 3.0517578125e-05f);
                const float xdt = st.act[j][ch];
                const float* Bv = &st.bc[j][sub * NSL];
#pragma unroll
                for (int i = 0; i < NSL; i += 2)
                    state_pair_fast(h[i], h[i + 1], bsl[i], bsl[i + 1], make_float2(ms, ms), make_float2(xdt, xdt),
                                    Bv[i], Bv[i + 1]);
                if (NSL % 4 == 0) {
#pragma unroll
                    for (int i = 0; i < NSL; i += 4)
                        *reinterpret_cast<float4*>(&snap[j][lane][i]) = make_float4(h[i], h[i + 1], h[i + 2], h[i + 3]);
                } else {
                    *reinterpret_cast<float2*>(&snap[j][lane][0]) = make_float2(h[0], h[1]);
                }
            }
        } else
#pragma unroll 1
        for (int j = 0; j < tn; j++) {
            const float mod = st.mod[j][ch];
            const float xdt = st.act[j][ch];
            const float* Bv = &st.bc[j][sub * NSL];
            if (fast_mask & (1u << j)) {
                const float ms = __fmul_rn(mod, 3.0517578125e-05f);
                // h = h * decay + (1 - decay) * u                       (:309)
#pragma unroll
                for (int i = 0; i < NSL; i += 2)
                    state_pair_fast(h[i], h[i + 1], bsl[i], bsl[i + 1], make_float2(ms, ms), make_float2(xdt, xdt),
                                    Bv[i], Bv[i + 1]);
            } else {
#pragma unroll
                for (int i = 0; i < NSL; i++) {
                    const float bn = __fmul_rn(bsl[i], 32768.0f);  // exact: back to base
                    const float num = ste_clamp(__fadd_rn(bn, mod), 0.0f, 32000.0f);
                    const float dec = __fmul_rn(num, 3.0517578125e-05f);
                    const float u = __fmul_rn(xdt, Bv[i]);
                    h[i] = __fadd_rn(__fmul_rn(h[i], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                }
            }
            if (NSL % 4 == 0) {
#pragma unroll
                for (int i = 0; i < NSL; i += 4)
                    *reinterpret_cast<float4*>(&snap[j][lane][i]) = make_float4(h[i], h[i + 1], h[i + 2], h[i + 3]);
            } else {
                *reinterpret_cast<float2*>(&snap[j][lane][0]) = make_float2(h[0], h[1]);
            }
        }
        __syncwarp();
        // (B2) y = matmul(h, C[..., None]): fused multiply-add over n = 0..15 from 0   (:440)
#pragma unroll
        for (int p = lane; p < SC * CHW; p += 32) {
            const int j = p / CHW, cc = p % CHW;
            if (j < tn) {
                const float* hs = &snap[j][cc * S][0];  // the 16 states of channel cc, n ascending
                const float* Cv = &st.bc[j][NS];
                float yacc = 0.0f;
#pragma unroll
                for (int n = 0; n < NS; n += 4) {
                    const float4 hq = *reinterpret_cast<const float4*>(hs + n);
                    const float4 cq = *reinterpret_cast<const float4*>(Cv + n);
                    yacc = __fmaf_rn(hq.x, cq.x, yacc);
                    yacc = __fmaf_rn(hq.y, cq.y, yacc);
                    yacc = __fmaf_rn(hq.z, cq.z, yacc);
                    yacc = __fmaf_rn(hq.w, cq.w, yacc);
                }
                st.mod[j][cc] = yacc;  // decay_mod of step j is no longer needed
            }
        }
        __syncwarp();
        // (C) gate, store, row absmax of steps j = sub + k*S               (:441-444)
        unsigned m[SPL];
#pragma unroll
        for (int k = 0; k < SPL; k++) {
            const int j = sub + k * S;
            const float out = sigmoid_gate(st.mod[j][ch], st.z[j][ch]);
            const bool ok = active && j < tn;
            if (ok) y[(row0 + t0 + j) * D + d] = out;
            m[k] = ok ? __float_as_uint(fabsf(out)) : 0u;
        }
        if (amax) {
            // reduce over the lanes of the same sub-index (xor offsets >= S keep it)
#pragma unroll
            for (int o = 16; o >= S; o >>= 1) {
#pragma unroll
                for (int k = 0; k < SPL; k++) m[k] = max(m[k], __shfl_xor_sync(0xffffffffu, m[k], o));
            }
            if (ch == 0) {
#pragma unroll
                for (int k = 0; k < SPL; k++) {
                    const int j = sub + k * S;
                    if (j < tn) atomicMax(reinterpret_cast<unsigned int*>(amax) + row0 + t0 + j, m[k]);
                }
            }
        }
        __syncwarp();  // the buffers are refilled by the next iteration
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    if (h_out && active) {
        // final states of the sequence [batch, D, 16] (the decode steps continue from them)
        float* dst = h_out + ((size_t)b * D + d) * NS + sub * NSL;
#pragma unroll
        for (int i = 0; i < NSL; i++) dst[i] = h[i];
    }
}

}  // namespace ssm
}  // namespace mi

extern "C" int mi_conv_act_quant(const float* xz, int ldx, const float* w, const float* bias, float* act, int8_t* xq,
                                 float* xscale, float* amax_ws, int batch, int L, int D, void* stream) {
    if (!xz || !w || !bias || !act) return MI_ERR_INVALID;
    if ((xq == nullptr) != (xscale == nullptr)) return MI_ERR_INVALID;
    if (xq && !amax_ws) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || D <= 0 || ldx < D) return MI_ERR_INVALID;
    if (((uintptr_t)w | (uintptr_t)bias | (uintptr_t)xz | (uintptr_t)act) & 15) return MI_ERR_INVALID;
    if ((D | ldx) & 3) return MI_ERR_UNSUPPORTED;  // 16-byte vectors of 4 channels
    if (batch > 65535 || mi::cdiv(L, mi::ssm::CONV_TC) > 65535) return MI_ERR_UNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    const int T = batch * L;
    if (amax_ws && cudaMemsetAsync(amax_ws, 0, sizeof(float) * (size_t)T, s) != cudaSuccess) return MI_ERR_CUDA;
    dim3 grid(mi::cdiv(D, 4 * mi::ssm::CONV_THREADS), batch, mi::cdiv(L, mi::ssm::CONV_TC));
    mi::ssm::conv_act_kernel<<<grid, mi::ssm::CONV_THREADS, 0, s>>>(
        xz, ldx, w, bias, act, reinterpret_cast<unsigned int*>(amax_ws), L, D);
    MI_CHECK_LAUNCH();
    if (xq) return mi_quantize_rows(act, D, T, D, xq, D, xscale, amax_ws, nullptr, stream);
    return MI_OK;
}

// mi_conv_act_quant with the row absmax and the quantisation inside the conv
// kernel (one CTA per chunk of whole rows): no workspace, one launch.
extern "C" int mi_conv_act_quant_rows(const float* xz, int ldx, const float* w, const float* bias, float* act,
                                      int8_t* xq, float* xscale, int batch, int L, int D, void* stream) {
    if (!xz || !w || !bias || !act || !xq || !xscale) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || D <= 0 || ldx < D) return MI_ERR_INVALID;
    if (((uintptr_t)w | (uintptr_t)bias | (uintptr_t)xz | (uintptr_t)act) & 15) return MI_ERR_INVALID;
    if (((uintptr_t)xq) & 3) return MI_ERR_INVALID;
    if ((D | ldx) & 3) return MI_ERR_UNSUPPORTED;  // 16-byte vectors of 4 channels
    if (D > 4096) return MI_ERR_UNSUPPORTED;       // D/4 threads per CTA
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    const int threads = mi::cdiv(D / 4, 32) * 32;
    dim3 grid(mi::cdiv(L, mi::ssm::CONV_TC), batch);
    const size_t ring = (size_t)mi::ssm::CONVR_RING * mi::ssm::CONVR_G * D * sizeof(float);
    // the ring: up to 72 KB (D <= 1536) / 192 KB (D <= 4096) of dynamic shared memory; the
    // attribute belongs to the current device's context, so it is set on every call
    if (cudaFuncSetAttribute(threads <= 384 ? (const void*)mi::ssm::conv_rows_kernel<384>
                                            : (const void*)mi::ssm::conv_rows_kernel<1024>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ring) != cudaSuccess) {
        cudaGetLastError();  // reported here; keep it out of later launch checks
        return MI_ERR_CUDA;
    }
    if (threads <= 384)
        MI_LAUNCH_DEPENDENT(mi::ssm::conv_rows_kernel<384>, grid, dim3(threads), ring, (cudaStream_t)stream, xz, ldx, w,
                            bias, act, xq, xscale, L, D);
    else
        MI_LAUNCH_DEPENDENT(mi::ssm::conv_rows_kernel<1024>, grid, dim3(threads), ring, (cudaStream_t)stream, xz, ldx,
                            w, bias, act, xq, xscale, L, D);
    return MI_OK;
}

namespace mi {
namespace ssm {

// Kernel choice: the pipelined kernel (ssm_scan_pipe_kernel), measured
// faster than one lane per channel (ssm_scan_kernel) and than 2, 4 or 8
// lanes (ssm_scan_split_kernel) at per-GPU batches 8, 16, 32 and 64 of the
// config-4 layer at 2048 tokens and level at 128 tokens; below 64 tokens (8
// chunks) its pipeline hardly fills and the one-lane kernel is faster
// (16 tokens x 256 sequences: 4.2 vs 5.3 ms per forward).  The others stay
// available by explicit request.
static int pick_split(int L) { return L >= 64 ? 3 : 1; }

template <int RW>
static void launch_scan(int split, int batch, int L, int D, const float* act, const float* bc, int ldbc,
                        const DtSource& src, const float* z, int ldz, const float* base, float* y, float* amax,
                        float* h_out, cudaStream_t s) {
    if (split == 3) {
        // 20 KB of shared memory per CTA: prefer the largest carveout so that registers bound
        // the residency (a per-context preference, set on every call like the others)
        cudaFuncSetAttribute(ssm_scan_pipe_kernel<RW>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
        dim3 grid(cdiv(D, 32), batch);
        // Not a dependent launch: launched early, the scan's CTAs are placed wherever the
        // previous kernel leaves room, and the uneven spread slows this latency-bound
        // grid when it is a single wave (per-GPU batch 8: 18.6 instead of 14.3 ms per
        // prefill step).
        ssm_scan_pipe_kernel<RW><<<grid, 128, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y, amax, h_out, L, D);
        return;
    }
    const int chw = SCAN_THREADS / split;
    dim3 grid(cdiv(D, chw), batch);
    if (split == 1)
        ssm_scan_kernel<RW, 1><<<grid, SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y, amax, h_out, L, D);
    else if (split == 2)
        ssm_scan_split_kernel<RW, 2><<<grid, SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y, amax, h_out,
                                                                   L, D);
    else if (split == 4)
        ssm_scan_split_kernel<RW, 4><<<grid, SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y, amax, h_out,
                                                                   L, D);
    else
        ssm_scan_split_kernel<RW, 8><<<grid, SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y, amax, h_out,
                                                                   L, D);
}

}  // namespace ssm
}  // namespace mi

extern "C" int mi_ssm_scan(const float* act, const float* bc, int ldbc, const float* modraw, const float* z, int ldz,
                           const float* base, float* y, float* amax, int batch, int L, int D, int N, void* stream) {
    if (!act || !bc || !modraw || !z || !base || !y) return MI_ERR_INVALID;
    if (N != mi::ssm::NS) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || L <= 0 || D <= 0 || ldbc < 2 * N || ldz < D) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    // 16-byte asynchronous staging of rows
    if (((uintptr_t)act | (uintptr_t)bc | (uintptr_t)modraw | (uintptr_t)z) & 15) return MI_ERR_UNSUPPORTED;
    if ((D | ldbc | ldz) & 3) return MI_ERR_UNSUPPORTED;
    mi::ssm::DtSource src{modraw, nullptr, 0, nullptr, nullptr, nullptr};
    mi::ssm::launch_scan<0>(mi::ssm::pick_split(L), batch, L, D, act, bc, ldbc, src, z, ldz, base, y, amax,
                            nullptr, (cudaStream_t)stream);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_ssm_scan_dt(const float* act, const float* bc, int ldbc, const int8_t* dtq, int ldq, const float* dts,
                              const int8_t* w_dt, const float* w_dt_scale, int R, const float* z, int ldz,
                              const float* base, float* y, float* amax, float* h_out, int batch, int L, int D, int N,
                              int split, void* stream) {
    if (!act || !bc || !dtq || !dts || !w_dt || !w_dt_scale || !z || !base || !y) return MI_ERR_INVALID;
    if (N != mi::ssm::NS) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || L <= 0 || D <= 0 || R <= 0 || ldbc < 2 * N || ldz < D) return MI_ERR_INVALID;
    if (split != 0 && split != 1 && split != 2 && split != 3 && split != 4 && split != 8) return MI_ERR_INVALID;
    const int R16 = (R + 15) / 16 * 16;
    if (R16 > 4 * mi::ssm::MAX_RW || ldq < R16 || (ldq & 15)) return MI_ERR_UNSUPPORTED;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)act | (uintptr_t)bc | (uintptr_t)z | (uintptr_t)dtq | (uintptr_t)w_dt) & 15)
        return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)dts) & 3) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)h_out) & 15) return MI_ERR_INVALID;
    if ((D | ldbc | ldz) & 3) return MI_ERR_UNSUPPORTED;
    if (split == 0) split = mi::ssm::pick_split(L);
    mi::ssm::DtSource src{nullptr, dtq, ldq, dts, w_dt, w_dt_scale};
    cudaStream_t s = (cudaStream_t)stream;
    switch (R16 / 4) {
        case 4: mi::ssm::launch_scan<4>(split, batch, L, D, act, bc, ldbc, src, z, ldz, base, y, amax, h_out, s); break;
        case 8: mi::ssm::launch_scan<8>(split, batch, L, D, act, bc, ldbc, src, z, ldz, base, y, amax, h_out, s); break;
        case 12: mi::ssm::launch_scan<12>(split, batch, L, D, act, bc, ldbc, src, z, ldz, base, y, amax, h_out, s); break;
        case 16: mi::ssm::launch_scan<16>(split, batch, L, D, act, bc, ldbc, src, z, ldz, base, y, amax, h_out, s); break;
        default: return MI_ERR_UNSUPPORTED;
    }
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
