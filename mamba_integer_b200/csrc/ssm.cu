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
// One thread per (sequence, channel) walks a chunk of CONV_TC positions with the
// 4-tap window in registers, so every input element is read once, coalesced
// across channels.  The row absmax needed by the following int8 quantisation
// is accumulated with one atomicMax per warp and position into amax (fp32
// bits of non-negative values order like unsigned integers; NaN sorts above
// +inf, which makes a NaN row propagate as torch.amax does).
constexpr int CONV_THREADS = 128;
constexpr int CONV_TC = 64;  // positions per CTA
constexpr int CONV_G = 8;    // positions per group: computed together, absmax reduced together

// xz: [batch*L, ldx], conv input = columns [0, D).  act: [batch*L, D].
__global__ void __launch_bounds__(CONV_THREADS)
conv_act_kernel(const float* __restrict__ xz, int ldx, const float* __restrict__ w, const float* __restrict__ bias,
                float* __restrict__ act, unsigned int* __restrict__ amax, int L, int D) {
    const int c = blockIdx.x * CONV_THREADS + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.y;
    const int t0 = blockIdx.z * CONV_TC;
    const bool active = c < D;
    const int cc = active ? c : 0;
    const float4 wc = *reinterpret_cast<const float4*>(w + 4 * cc);
    const float bs = bias[cc];
    const size_t row0 = (size_t)b * L;
    const float* px = xz + row0 * ldx + cc;
    // window x[t-3], x[t-2], x[t-1]
    float w0 = (t0 - 3 >= 0) ? px[(size_t)(t0 - 3) * ldx] : 0.0f;
    float w1 = (t0 - 2 >= 0) ? px[(size_t)(t0 - 2) * ldx] : 0.0f;
    float w2 = (t0 - 1 >= 0) ? px[(size_t)(t0 - 1) * ldx] : 0.0f;
    const int tend = min(L, t0 + CONV_TC);
    for (int t = t0; t < tend; t += CONV_G) {
        float xv[CONV_G];
#pragma unroll
        for (int j = 0; j < CONV_G; j++) xv[j] = (t + j < tend) ? __ldg(px + (size_t)(t + j) * ldx) : 0.0f;
        unsigned m[CONV_G];
#pragma unroll
        for (int j = 0; j < CONV_G; j++) {
            // bias first, then one FMA per tap k = 0..3 over positions t-3+k
            float acc = bs;
            acc = __fmaf_rn(wc.x, w0, acc);
            acc = __fmaf_rn(wc.y, w1, acc);
            acc = __fmaf_rn(wc.z, w2, acc);
            acc = __fmaf_rn(wc.w, xv[j], acc);
            w0 = w1;
            w1 = w2;
            w2 = xv[j];
            const float a = squareplus(ste_clamp(acc, -50.0f, 50.0f));
            const bool ok = active && (t + j < tend);
            if (ok) act[(row0 + t + j) * D + c] = a;
            m[j] = ok ? __float_as_uint(fabsf(a)) : 0u;
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
template <int RW>
__device__ __forceinline__ void scan_stage_load(ScanStage& st, const float* __restrict__ act, const DtSource& src,
                                                const float* __restrict__ z, const float* __restrict__ bc, int ldbc,
                                                int ldz, size_t row0, int t0, int L, int d0, int D) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int h2 = 0; h2 < SC * 8 / 32; h2++) {
        const int idx = lane + 32 * h2;  // 16-byte chunk: step r, quarter q
        const int r = idx >> 3, q = idx & 7;
        const int t = t0 + r;
        const bool okt = t < L;
        const bool ok = okt && (d0 + 4 * q < D);
        const size_t row = row0 + (okt ? t : 0);
        const int c = d0 + (ok ? 4 * q : 0);
        cp_async16(&st.act[r][4 * q], act + row * D + c, ok);
        if (RW == 0) cp_async16(&st.mod[r][4 * q], src.modraw + row * D + c, ok);
        cp_async16(&st.z[r][4 * q], z + row * ldz + c, ok);
        cp_async16(&st.bc[r][4 * q], bc + row * ldbc + (okt ? 4 * q : 0), okt);
    }
    if (RW > 0) {
        // dt rows: SC rows x (RW/4) chunks of 16 bytes; scales: SC x 4 bytes
        for (int idx = lane; idx < SC * (RW / 4); idx += 32) {
            const int r = idx / (RW / 4), q = idx % (RW / 4);
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

// One warp owns 32 channels of one sequence; each lane carries its channel's
// 16 fp32 states in registers for the whole sequence.  Inputs arrive through
// a per-warp double-buffered cp.async ring of SC-step chunks (no block-level
// barriers).  Each chunk is processed in three phases so that only the state
// recurrence is serial: (A) decay clamp / dt / x*dt for SC steps, (B) the
// 16-state convex update and h.C per step, (C) gates, stores and the row
// absmax reductions for SC steps at once.
//
// RW > 0 fuses the dt_proj BitLinear: each lane keeps its channel's ternary
// dt_proj weights (4*RW int8) in registers and forms the exact int32 dot
// product with the step's quantised dt row by dp4a, then applies the
// BitLinear rescale acc * (w_scale * dt_scale[t]) exactly as the GEMM
// epilogue does (src/rational_bitnet.py:204-208).
// (22 one-warp CTAs per SM by registers and shared memory: all 3072 CTAs of a
// 64-sequence x 1536-channel layer are resident at once.)
template <int RW>
__global__ void __launch_bounds__(SCAN_THREADS, 22)
ssm_scan_kernel(const float* __restrict__ act, const float* __restrict__ bc, int ldbc, const DtSource src,
                const float* __restrict__ z, int ldz, const float* __restrict__ base, float* __restrict__ y,
                float* __restrict__ amax, int L, int D) {
    __shared__ __align__(16) ScanStage stage[SSTAGES];
    const int lane = threadIdx.x;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * 32;
    const int d = d0 + lane;
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

    // states and base / 2^15 in pairs for the packed f32x2 arithmetic
    float2 h2[NS / 2], bs2[NS / 2];
    float bmin = __int_as_float(0x7f800000), bmax = -__int_as_float(0x7f800000);
    bool bnan = false;
#pragma unroll
    for (int i = 0; i < NS / 2; i++) {
        const float b0 = base[(size_t)dd * NS + 2 * i], b1 = base[(size_t)dd * NS + 2 * i + 1];
        bs2[i] = make_float2(__fmul_rn(b0, 3.0517578125e-05f), __fmul_rn(b1, 3.0517578125e-05f));
        h2[i] = make_float2(0.0f, 0.0f);
        bmin = fminf(bmin, fminf(b0, b1));
        bmax = fmaxf(bmax, fmaxf(b0, b1));
        bnan |= (b0 != b0) | (b1 != b1);
    }

    const int nchunks = cdiv(L, SC);
    scan_stage_load<RW>(stage[0], act, src, z, bc, ldbc, ldz, row0, 0, L, d0, D);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int c = 0; c < nchunks; c++) {
        ScanStage& st = stage[c & 1];
        if (c + 1 < nchunks)
            scan_stage_load<RW>(stage[(c + 1) & 1], act, src, z, bc, ldbc, ldz, row0, (c + 1) * SC, L, d0, D);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncwarp();
        const int t0 = c * SC;
        const int tn = min(SC, L - t0);
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
                st.mod[j][lane] = __fmul_rn((float)acc, __fmul_rn(wsc, st.dts[j]));
            }
        }

        // (A) per (step, channel): decay_mod, dt_val, x*dt   (:419-428)
        unsigned fast_mask = 0;
#pragma unroll
        for (int j = 0; j < SC; j++) {
            const float mod = ste_clamp(st.mod[j][lane], -20.0f, 20.0f);
            const float dtv = ste_clamp(__fmul_rn(squareplus(mod), 0.01f), 0.001f, 0.1f);
            st.mod[j][lane] = mod;
            st.act[j][lane] = __fmul_rn(st.act[j][lane], dtv);  // x * dt_val
            // decay_nums = ste_clamp(v, 0, 32000), v = base + mod, equals the plain
            // clamp(v, 0, 32000) whenever v <= 64000: for v > 32000 the difference
            // 32000 - v is exact (Sterbenz) so v + (32000 - v) = 32000, for v < 0 it
            // gives +0, and inside the range it is the identity.  Rounding is monotone,
            // so the channel's largest base decides.  base >= 1 and a mod that is 0 or
            // not tiny keep base/2^15 and mod/2^15 exact (no subnormals), which the
            // fast path below relies on.
            const bool inside = !bnan && (bmin >= 1.0f) && (__fadd_rn(bmax, mod) <= 64000.0f) &&
                                (mod == 0.0f || fabsf(mod) >= 1e-30f);
            if (__all_sync(0xffffffffu, inside)) fast_mask |= 1u << j;
        }
        // (B) the recurrence, one step at a time
#pragma unroll 1
        for (int j = 0; j < tn; j++) {
            const float mod = st.mod[j][lane];
            const float xdt = st.act[j][lane];
            const float2* B2 = reinterpret_cast<const float2*>(&st.bc[j][0]);
            const float2* C2 = reinterpret_cast<const float2*>(&st.bc[j][NS]);
            if (fast_mask & (1u << j)) {
                // decay = clamp(base + mod, 0, 32000) / 2^15
                //       = clamp(base/2^15 + mod/2^15, 0, 32000/2^15): both scalings are
                // exact, the sum rounds once, and scaling by 2^-15 commutes with
                // rounding and with the clamp away from subnormals
                const float ms = __fmul_rn(mod, 3.0517578125e-05f);
#pragma unroll
                for (int i = 0; i < NS / 2; i++) {
                    const float2 bq = B2[i];
                    float hv[2] = {h2[i].x, h2[i].y};
                    const float bb[2] = {bs2[i].x, bs2[i].y}, Bq[2] = {bq.x, bq.y};
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const float dec = clamp_t(__fadd_rn(bb[e], ms), 0.0f, 0.9765625f);  // 32000 / 2^15
                        const float u = __fmul_rn(xdt, Bq[e]);
                        // h = h * decay + (1 - decay) * u                   (:309)
                        hv[e] = __fadd_rn(__fmul_rn(hv[e], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                    }
                    h2[i] = make_float2(hv[0], hv[1]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < NS / 2; i++) {
                    const float2 bq = B2[i];
                    float hv[2] = {h2[i].x, h2[i].y};
                    const float bb[2] = {bs2[i].x, bs2[i].y}, Bq[2] = {bq.x, bq.y};
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const float bn = __fmul_rn(bb[e], 32768.0f);  // exact: back to base
                        const float num = ste_clamp(__fadd_rn(bn, mod), 0.0f, 32000.0f);
                        const float dec = __fmul_rn(num, 3.0517578125e-05f);
                        const float u = __fmul_rn(xdt, Bq[e]);
                        hv[e] = __fadd_rn(__fmul_rn(hv[e], dec), __fmul_rn(__fsub_rn(1.0f, dec), u));
                    }
                    h2[i] = make_float2(hv[0], hv[1]);
                }
            }
            // y = matmul(h, C[..., None]): fused multiply-add over n = 0..15 from 0   (:440)
            float yacc = 0.0f;
#pragma unroll
            for (int i = 0; i < NS / 2; i++) {
                const float2 cq = C2[i];
                yacc = __fmaf_rn(h2[i].x, cq.x, yacc);
                yacc = __fmaf_rn(h2[i].y, cq.y, yacc);
            }
            st.mod[j][lane] = yacc;  // decay_mod of step j is no longer needed
        }
        // (C) gate, store, row absmax                                 (:441-444)
        unsigned m[SC];
#pragma unroll
        for (int j = 0; j < SC; j++) {
            const float out = sigmoid_gate(st.mod[j][lane], st.z[j][lane]);
            if (j < tn && active) y[(row0 + t0 + j) * D + d] = out;
            m[j] = (j < tn && active) ? __float_as_uint(fabsf(out)) : 0u;
        }
        if (amax) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
                for (int j = 0; j < SC; j++) m[j] = max(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
            }
            // fp32 bits of non-negative values order like unsigned ints (NaN above +inf)
            unsigned mine = 0u;  // lane j publishes step j
#pragma unroll
            for (int j = 0; j < SC; j++) mine = (lane == j) ? m[j] : mine;
            if (lane < tn) atomicMax(reinterpret_cast<unsigned int*>(amax) + row0 + t0 + lane, mine);
        }
        __syncwarp();  // the buffer is refilled by the next iteration's copies
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

}  // namespace ssm
}  // namespace mi

extern "C" int mi_conv_act_quant(const float* xz, int ldx, const float* w, const float* bias, float* act, int8_t* xq,
                                 float* xscale, float* amax_ws, int batch, int L, int D, void* stream) {
    if (!xz || !w || !bias || !act) return MI_ERR_INVALID;
    if ((xq == nullptr) != (xscale == nullptr)) return MI_ERR_INVALID;
    if (xq && !amax_ws) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || D <= 0 || ldx < D) return MI_ERR_INVALID;
    if (((uintptr_t)w) & 15) return MI_ERR_INVALID;
    if (batch > 65535 || mi::cdiv(L, mi::ssm::CONV_TC) > 65535) return MI_ERR_UNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    const int T = batch * L;
    if (amax_ws && cudaMemsetAsync(amax_ws, 0, sizeof(float) * (size_t)T, s) != cudaSuccess) return MI_ERR_CUDA;
    dim3 grid(mi::cdiv(D, mi::ssm::CONV_THREADS), batch, mi::cdiv(L, mi::ssm::CONV_TC));
    mi::ssm::conv_act_kernel<<<grid, mi::ssm::CONV_THREADS, 0, s>>>(
        xz, ldx, w, bias, act, reinterpret_cast<unsigned int*>(amax_ws), L, D);
    MI_CHECK_LAUNCH();
    if (xq) return mi_quantize_rows(act, D, T, D, xq, D, xscale, amax_ws, stream);
    return MI_OK;
}

extern "C" int mi_ssm_scan(const float* act, const float* bc, int ldbc, const float* modraw, const float* z, int ldz,
                           const float* base, float* y, float* amax, int batch, int L, int D, int N, void* stream) {
    if (!act || !bc || !modraw || !z || !base || !y) return MI_ERR_INVALID;
    if (N != mi::ssm::NS) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || L <= 0 || D <= 0 || ldbc < 2 * N || ldz < D) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    // 16-byte asynchronous staging of rows
    if (((uintptr_t)act | (uintptr_t)bc | (uintptr_t)modraw | (uintptr_t)z) & 15) return MI_ERR_UNSUPPORTED;
    if ((D | ldbc | ldz) & 3) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(D, mi::ssm::SCAN_THREADS), batch);
    mi::ssm::DtSource src{modraw, nullptr, 0, nullptr, nullptr, nullptr};
    mi::ssm::ssm_scan_kernel<0><<<grid, mi::ssm::SCAN_THREADS, 0, (cudaStream_t)stream>>>(act, bc, ldbc, src, z, ldz,
                                                                                          base, y, amax, L, D);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_ssm_scan_dt(const float* act, const float* bc, int ldbc, const int8_t* dtq, int ldq, const float* dts,
                              const int8_t* w_dt, const float* w_dt_scale, int R, const float* z, int ldz,
                              const float* base, float* y, float* amax, int batch, int L, int D, int N, void* stream) {
    if (!act || !bc || !dtq || !dts || !w_dt || !w_dt_scale || !z || !base || !y) return MI_ERR_INVALID;
    if (N != mi::ssm::NS) return MI_ERR_UNSUPPORTED;
    if (batch <= 0 || L <= 0 || D <= 0 || R <= 0 || ldbc < 2 * N || ldz < D) return MI_ERR_INVALID;
    const int R16 = (R + 15) / 16 * 16;
    if (R16 > 4 * mi::ssm::MAX_RW || ldq < R16 || (ldq & 15)) return MI_ERR_UNSUPPORTED;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)act | (uintptr_t)bc | (uintptr_t)z | (uintptr_t)dtq | (uintptr_t)w_dt) & 15)
        return MI_ERR_UNSUPPORTED;
    if (((uintptr_t)dts) & 3) return MI_ERR_UNSUPPORTED;
    if ((D | ldbc | ldz) & 3) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(D, mi::ssm::SCAN_THREADS), batch);
    mi::ssm::DtSource src{nullptr, dtq, ldq, dts, w_dt, w_dt_scale};
    cudaStream_t s = (cudaStream_t)stream;
    switch (R16 / 4) {
        case 4:
            mi::ssm::ssm_scan_kernel<4><<<grid, mi::ssm::SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y,
                                                                                amax, L, D);
            break;
        case 8:
            mi::ssm::ssm_scan_kernel<8><<<grid, mi::ssm::SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y,
                                                                                amax, L, D);
            break;
        case 12:
            mi::ssm::ssm_scan_kernel<12><<<grid, mi::ssm::SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y,
                                                                                 amax, L, D);
            break;
        case 16:
            mi::ssm::ssm_scan_kernel<16><<<grid, mi::ssm::SCAN_THREADS, 0, s>>>(act, bc, ldbc, src, z, ldz, base, y,
                                                                                 amax, L, D);
            break;
        default:
            return MI_ERR_UNSUPPORTED;
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
