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
// Layout / parallelism: one warp per CTA owns 16 channels of one sequence;
// two lanes per channel each hold 8 of the 16 int32 states in registers for
// the whole sequence (the recurrence is sequential in t).  x and B|C arrive
// through a per-warp double-buffered cp.async ring of TC-step chunks (no
// block-level barriers); the two half sums of y meet with one shuffle, y is
// staged in shared memory and written as 16-byte vectors.  n stays in
// registers.
//
// Exactness: the shifted product fits int32 whenever 0 <= n <= 2^k (so the
// 64-bit shift result is truncated losslessly); |B*x| < 2^30 when
// |B|,|x| <= 32767; the state add is checked for int32 overflow with a sign
// test and y is accumulated in 64 bits.  Violations set the device error word
// instead of producing wrong values silently.
#include "mi_common.cuh"

namespace mi {
namespace scan_i32 {

constexpr int CH = 16;       // channels per warp
constexpr int THREADS = 32;  // two lanes per channel
constexpr int TC = 16;       // time steps per staged chunk
constexpr int NS = 16;       // d_state
constexpr int HALF = NS / 2;

struct Stage {
    int32_t x[TC][CH];
    int32_t bc[TC][2 * NS];  // B[0..15] | C[0..15]
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(pred ? 16 : 0)
                 : "memory");
}

// Stage chunk [t0, t0+TC) of x[b, :, d0:d0+CH] and B|C[b, :, :].
__device__ __forceinline__ void load_chunk(Stage& st, int t0, const int32_t* __restrict__ x,
                                           const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                                           size_t row0, int d0, int L, int D) {
    const int lane = threadIdx.x;
#pragma unroll
    for (int i = lane; i < TC * (CH / 4); i += 32) {  // x: TC rows x 4 chunks
        const int r = i >> 2, q = i & 3;
        const int t = t0 + r;
        const bool ok = (t < L) && (d0 + 4 * q < D);
        const int32_t* src = ok ? x + (row0 + t) * D + d0 + 4 * q : x;
        cp_async16(&st.x[r][4 * q], src, ok);
    }
#pragma unroll
    for (int i = lane; i < TC * 8; i += 32) {  // B|C: TC rows x 8 chunks
        const int r = i >> 3, q = i & 7;
        const int t = t0 + r;
        const bool ok = t < L;
        const int32_t* base = (q < 4) ? Bm : Cm;
        const int32_t* src = ok ? base + (row0 + t) * NS + (q & 3) * 4 : base;
        cp_async16(&st.bc[r][4 * q], src, ok);
    }
}

template <bool Y64>
__global__ void __launch_bounds__(THREADS)
scan_i32_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                const int32_t* __restrict__ n, int k, int32_t* __restrict__ y32, int64_t* __restrict__ y64,
                int32_t* __restrict__ h_io, int L, int D) {
    __shared__ __align__(16) Stage stage[2];
    __shared__ __align__(16) int64_t ys[TC][CH];
    const int lane = threadIdx.x;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CH;
    const int ch = lane >> 1;   // channel within the warp
    const int half = lane & 1;  // which 8 states
    const int d = d0 + ch;
    const bool active = d < D;
    const size_t row0 = (size_t)b * L;

    int32_t h[HALF], nn[HALF];
    int bad = 0;
    const int32_t lim = 1 << k;
#pragma unroll
    for (int j = 0; j < HALF; j++) {
        const int jj = half * HALF + j;
        h[j] = active ? h_io[((size_t)b * D + d) * NS + jj] : 0;
        nn[j] = active ? n[(size_t)d * NS + jj] : 0;
        bad |= (nn[j] < 0) | (nn[j] > lim);
    }

    int ovf = 0;  // sign-test accumulator: negative => an int32 state or y32 overflowed
    const int nchunks = cdiv(L, TC);
    load_chunk(stage[0], 0, x, Bm, Cm, row0, d0, L, D);
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int c = 0; c < nchunks; c++) {
        Stage& st = stage[c & 1];
        if (c + 1 < nchunks) load_chunk(stage[(c + 1) & 1], (c + 1) * TC, x, Bm, Cm, row0, d0, L, D);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncwarp();
        // range check of the staged inputs: 24 values per lane per chunk
#pragma unroll
        for (int i = lane; i < TC * CH; i += 32) {
            const int32_t v = (&st.x[0][0])[i];
            bad |= (v < -32767) | (v > 32767);
        }
#pragma unroll
        for (int i = lane; i < TC * 2 * NS; i += 32) {
            const int32_t v = (&st.bc[0][0])[i];
            bad |= (v < -32767) | (v > 32767);
        }
        const int t0 = c * TC;
        const int tn = min(TC, L - t0);
#pragma unroll 2
        for (int r = 0; r < tn; r++) {
            const int32_t xv = st.x[r][ch];
            const int4 b0 = *reinterpret_cast<const int4*>(&st.bc[r][half * HALF]);
            const int4 b1 = *reinterpret_cast<const int4*>(&st.bc[r][half * HALF + 4]);
            const int4 c0 = *reinterpret_cast<const int4*>(&st.bc[r][NS + half * HALF]);
            const int4 c1 = *reinterpret_cast<const int4*>(&st.bc[r][NS + half * HALF + 4]);
            const int32_t bb[HALF] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            const int32_t cc[HALF] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            // the 8 state chains are independent; the integer sums below are exact
            // in any order, so they are formed as trees to keep dependency chains short
            long long prod[HALF];
            int32_t ov[HALF];
#pragma unroll
            for (int j = 0; j < HALF; j++) {
                const long long p = (long long)h[j] * (long long)nn[j];
                const int32_t s = (int32_t)(p >> k);
                const int32_t bx = (int32_t)((uint32_t)bb[j] * (uint32_t)xv);  // |B*x| < 2^30 when in range
                const int32_t hn = (int32_t)((uint32_t)s + (uint32_t)bx);
                ov[j] = (s ^ hn) & (bx ^ hn);
                h[j] = hn;
                prod[j] = (long long)cc[j] * (long long)hn;
            }
            ovf |= ((ov[0] | ov[1]) | (ov[2] | ov[3])) | ((ov[4] | ov[5]) | (ov[6] | ov[7]));
            long long acc = ((prod[0] + prod[1]) + (prod[2] + prod[3])) + ((prod[4] + prod[5]) + (prod[6] + prod[7]));
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            if (half == 0) ys[r][ch] = acc;
        }
        __syncwarp();
        // write the chunk's y rows: TC rows x CH values as 16-byte vectors
        if (Y64) {
            for (int i = lane; i < TC * (CH / 2); i += 32) {
                const int r = i >> 3, q = i & 7;  // 8 chunks of two int64 per row
                const int dq = d0 + 2 * q;
                if (r < tn && dq < D) {
                    int64_t* o = y64 + (row0 + t0 + r) * D + dq;
                    *reinterpret_cast<longlong2*>(o) = make_longlong2(ys[r][2 * q], ys[r][2 * q + 1]);
                }
            }
        } else {
            for (int i = lane; i < TC * (CH / 4); i += 32) {
                const int r = i >> 2, q = i & 3;  // 4 chunks of four int32 per row
                const int dq = d0 + 4 * q;
                if (r < tn && dq < D) {
                    int32_t v[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const long long a = ys[r][4 * q + e];
                        if (a > INT32_MAX || a < INT32_MIN) ovf |= INT32_MIN;
                        v[e] = (int32_t)a;
                    }
                    *reinterpret_cast<int4*>(y32 + (row0 + t0 + r) * D + dq) = make_int4(v[0], v[1], v[2], v[3]);
                }
            }
        }
        __syncwarp();  // ys and the stage buffer are rewritten next iteration
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");

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
    if (D % 4 != 0) return MI_ERR_UNSUPPORTED;  // 16-byte staging of x rows and vector y stores
    if (((uintptr_t)x | (uintptr_t)B | (uintptr_t)C | (uintptr_t)y32 | (uintptr_t)y64) & 15) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(D, CH), batch);
    cudaStream_t s = (cudaStream_t)stream;
    if (y64)
        scan_i32_kernel<true><<<grid, THREADS, 0, s>>>(x, B, C, n, k, nullptr, y64, h_io, L, D);
    else
        scan_i32_kernel<false><<<grid, THREADS, 0, s>>>(x, B, C, n, k, y32, nullptr, h_io, L, D);
    MI_CHECK_LAUNCH();
    return MI_OK;
}
