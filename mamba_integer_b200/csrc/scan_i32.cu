// scan_i32.cu -- integer dyadic selective scan (sm_100a).
//
//   h[b,d,j] <- ((int64)h * n[d,j]) >> k  +  B[b,t,j] * x[b,t,d]
//   y[b,t,d]  = sum_j C[b,t,j] * h[b,d,j]
//
// The state update follows the reference POC kernel
// (src/cuda_kernels/dyadic_mamba_kernel.cu:53-59: 64-bit product, arithmetic
// right shift, add) with the selective-scan input term B_t*x_t and the output
// contraction C_t.h_t added.
//
// Layout / parallelism: one CTA per (batch row b, block of 64 channels); two
// threads per channel, each holding 8 of the 16 states in registers for the
// whole sequence (the recurrence is sequential in t).  x, B and C are staged
// through a 3-deep shared-memory ring of 32-step chunks with cp.async so the
// HBM reads run ahead of the arithmetic; y is combined across the two halves
// with one shuffle and written per step.  n stays in registers.
//
// Exactness: the shifted product fits int32 whenever 0 <= n <= 2^k (so the
// 64-bit shift result is truncated losslessly); |B*x| < 2^30 when
// |B|,|x| <= 32767; the state add is checked for int32 overflow with a
// sign test, y is accumulated in 64 bits.  Violations set the device error
// word instead of producing wrong values silently.
#include "mi_common.cuh"

namespace mi {
namespace scan_i32 {

constexpr int CH = 64;          // channels per CTA
constexpr int THREADS = 2 * CH; // two state halves per channel
constexpr int TC = 32;          // time steps per staged chunk
constexpr int STAGES = 3;
constexpr int NS = 16;          // d_state
constexpr int HALF = NS / 2;

struct Smem {
    int32_t x[STAGES][TC][CH];
    int32_t bc[STAGES][TC][2 * NS];  // B[0..15] | C[0..15]
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    int sz = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(sz));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Stage chunk `c` (steps [c*TC, c*TC+TC)) of x[b, :, d0:d0+CH] and B/C[b, :, :].
__device__ __forceinline__ void load_chunk(Smem& sm, int stage, int c, const int32_t* __restrict__ x,
                                           const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                                           int b, int d0, int L, int D) {
    const int tid = threadIdx.x;
    // x: TC rows x CH int32 = TC*16 chunks of 16 B
    for (int i = tid; i < TC * (CH / 4); i += THREADS) {
        int r = i / (CH / 4), q = i % (CH / 4);
        int t = c * TC + r;
        int d = d0 + q * 4;
        bool ok = (t < L) && (d < D);
        const int32_t* src = ok ? x + ((size_t)b * L + t) * D + d : x;
        cp_async16(&sm.x[stage][r][q * 4], src, ok);
    }
    // B and C: TC rows x 16 int32 each = 4 chunks per row per matrix
    for (int i = tid; i < TC * 8; i += THREADS) {
        int r = i / 8, q = i % 8;
        int t = c * TC + r;
        bool ok = t < L;
        const int32_t* base = (q < 4) ? Bm : Cm;
        const int32_t* src = ok ? base + ((size_t)b * L + t) * NS + (q & 3) * 4 : base;
        cp_async16(&sm.bc[stage][r][(q >> 2) * NS + (q & 3) * 4], src, ok);
    }
}

template <bool Y64>
__global__ void __launch_bounds__(THREADS)
scan_i32_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                const int32_t* __restrict__ n, int k, int32_t* __restrict__ y32, int64_t* __restrict__ y64,
                int32_t* __restrict__ h_io, int L, int D) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CH;
    const int tid = threadIdx.x;
    const int ch = tid >> 1;         // channel within the CTA
    const int half = tid & 1;        // which 8 states
    const int d = d0 + ch;
    const bool active = d < D;

    int32_t h[HALF];
    int32_t nn[HALF];
    int bad = 0;
    const int32_t lim = 1 << k;
#pragma unroll
    for (int j = 0; j < HALF; j++) {
        int jj = half * HALF + j;
        h[j] = active ? h_io[((size_t)b * D + d) * NS + jj] : 0;
        nn[j] = active ? n[(size_t)d * NS + jj] : 0;
        bad |= (nn[j] < 0) | (nn[j] > lim);
    }

    const int nchunks = cdiv(L, TC);
#pragma unroll
    for (int s = 0; s < STAGES - 1; s++) {
        if (s < nchunks) load_chunk(sm, s, s, x, Bm, Cm, b, d0, L, D);
        cp_async_commit();
    }

    int ovf = 0;  // sign-test accumulator: negative => an int32 state overflowed
    for (int c = 0; c < nchunks; c++) {
        // keep STAGES-1 chunks in flight
        int cn = c + STAGES - 1;
        if (cn < nchunks) load_chunk(sm, cn % STAGES, cn, x, Bm, Cm, b, d0, L, D);
        cp_async_commit();
        cp_async_wait<STAGES - 1>();
        __syncthreads();
        const int st = c % STAGES;
        // range check of the staged inputs (cheap: a few values per thread per chunk)
        for (int i = tid; i < TC * CH; i += THREADS) {
            int32_t v = (&sm.x[st][0][0])[i];
            bad |= (v < -32767) | (v > 32767);
        }
        for (int i = tid; i < TC * 2 * NS; i += THREADS) {
            int32_t v = (&sm.bc[st][0][0])[i];
            bad |= (v < -32767) | (v > 32767);
        }
        const int tmax = min(TC, L - c * TC);
        for (int r = 0; r < tmax; r++) {
            const int32_t xv = sm.x[st][r][ch];
            const int32_t* Bv = &sm.bc[st][r][half * HALF];
            const int32_t* Cv = &sm.bc[st][r][NS + half * HALF];
            int4 b0 = *reinterpret_cast<const int4*>(Bv);
            int4 b1 = *reinterpret_cast<const int4*>(Bv + 4);
            int4 c0 = *reinterpret_cast<const int4*>(Cv);
            int4 c1 = *reinterpret_cast<const int4*>(Cv + 4);
            const int32_t bb[HALF] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            const int32_t cc[HALF] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            long long acc = 0;
#pragma unroll
            for (int j = 0; j < HALF; j++) {
                long long p = (long long)h[j] * (long long)nn[j];
                int32_t s = (int32_t)(p >> k);
                int32_t bx = (int32_t)((uint32_t)bb[j] * (uint32_t)xv);  // |B*x| < 2^30 when in range
                int32_t hn = (int32_t)((uint32_t)s + (uint32_t)bx);
                ovf |= (s ^ hn) & (bx ^ hn);
                h[j] = hn;
                acc += (long long)cc[j] * (long long)hn;
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            if (active && half == 0) {
                size_t o = ((size_t)b * L + (size_t)c * TC + r) * D + d;
                if (Y64) {
                    y64[o] = acc;
                } else {
                    if (acc > INT32_MAX || acc < INT32_MIN) ovf |= INT32_MIN;
                    y32[o] = (int32_t)acc;
                }
            }
        }
        __syncthreads();  // stage st is refilled by the next iteration's load
    }
    cp_async_wait<0>();

    if (active) {
#pragma unroll
        for (int j = 0; j < HALF; j++) h_io[((size_t)b * D + d) * NS + half * HALF + j] = h[j];
    }
    if (ovf < 0) raise_dev_error(MI_DEV_OVERFLOW);
    if (bad) raise_dev_error(MI_DEV_PRECOND);
}

}  // namespace scan_i32
}  // namespace mi

extern "C" int mi_scan_i32(const int32_t* x, const int32_t* B, const int32_t* C, const int32_t* n, int k,
                           int32_t* y32, int64_t* y64, int32_t* h_io, int batch, int L, int D, int N,
                           void* stream) {
    using namespace mi::scan_i32;
    if (!x || !B || !C || !n || !h_io) return MI_ERR_INVALID;
    if ((y32 == nullptr) == (y64 == nullptr)) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || D <= 0) return MI_ERR_INVALID;
    if (N != NS) return MI_ERR_UNSUPPORTED;
    if (k < 1 || k > 30) return MI_ERR_UNSUPPORTED;
    if (D % 4 != 0) return MI_ERR_UNSUPPORTED;  // 16-byte staging of x rows
    if (((uintptr_t)x | (uintptr_t)B | (uintptr_t)C) & 15) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(D, CH), batch);
    size_t smem = sizeof(Smem);
    cudaStream_t s = (cudaStream_t)stream;
    if (y64) {
        cudaFuncSetAttribute(scan_i32_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        scan_i32_kernel<true><<<grid, THREADS, smem, s>>>(x, B, C, n, k, nullptr, y64, h_io, L, D);
    } else {
        cudaFuncSetAttribute(scan_i32_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        scan_i32_kernel<false><<<grid, THREADS, smem, s>>>(x, B, C, n, k, y32, nullptr, h_io, L, D);
    }
    MI_CHECK_LAUNCH();
    return MI_OK;
}
