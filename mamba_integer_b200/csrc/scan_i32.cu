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
// Layout / parallelism: one warp per CTA owns 32/LPC channels of one
// sequence; LPC lanes per channel each hold 16/LPC of the 16 int32 states in
// registers for the whole sequence (the recurrence is sequential in t, so the
// independent (sequence, channel, state) chains are all the parallelism there
// is).  x and B|C arrive through a per-warp 4-deep cp.async ring of TC-step
// chunks (three chunks in flight ahead of the one in use, no block-level
// barriers).  Each lane folds its states' C*h into y with 64-bit
// multiply-adds, the LPC partial sums meet in shuffles, y is staged in shared
// memory and written as 16-byte vectors.  n stays in registers.  LPC = 2 at
// config 2 sizes: the B|C values every lane must receive each step (a 16-byte
// shared load delivers 512 bytes per warp) and the y shuffles share one
// load/store data path, which fewer lanes per channel use less of per state
// update.
//
// Exactness: the shifted product fits int32 whenever 0 <= n <= 2^k (so the
// 64-bit shift result is truncated losslessly); |B*x| < 2^30 when
// |B|,|x| <= 32767; the state add is checked for int32 overflow with a sign
// test and y is accumulated in 64 bits.  Violations set the device error word
// instead of producing wrong values silently.
#include "mi_common.cuh"

namespace mi {
namespace scan_i32 {

constexpr int NS = 16;       // d_state
constexpr int THREADS = 32;
constexpr int TC = 16;       // time steps per staged chunk
constexpr int SST = 4;       // chunks in the ring (SST - 1 in flight ahead)

template <int LPC>
struct Geo {
    static constexpr int SPL = NS / LPC;  // states per lane
    static constexpr int CH = 32 / LPC;   // channels per warp
    static constexpr int XQ = CH / 4;     // 16-byte chunks per staged x row
};

template <int CH>
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
template <int CH>
__device__ __forceinline__ void load_chunk(Stage<CH>& st, int t0, const int32_t* __restrict__ x,
                                           const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                                           size_t row0, int d0, int L, int D) {
    constexpr int XQ = CH / 4;
    const int lane = threadIdx.x;
#pragma unroll
    for (int i = lane; i < TC * XQ; i += 32) {
        const int r = i / XQ, q = i % XQ;
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

__device__ __forceinline__ int out_of_range4(int4 v) {
    // |v| > 32767 for any component (the preconditions of the exact int32 path)
    return ((unsigned)v.x + 32767u > 65534u) | ((unsigned)v.y + 32767u > 65534u) |
           ((unsigned)v.z + 32767u > 65534u) | ((unsigned)v.w + 32767u > 65534u);
}

template <int LPC, bool Y64>
__global__ void __launch_bounds__(THREADS)
scan_i32_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                const int32_t* __restrict__ n, int k, int32_t* __restrict__ y32, int64_t* __restrict__ y64,
                int32_t* __restrict__ h_io, int L, int D) {
    using G = Geo<LPC>;
    constexpr int SPL = G::SPL, CH = G::CH;
    __shared__ __align__(16) Stage<CH> stage[SST];
    __shared__ __align__(16) int64_t ys[TC][CH];
    const int lane = threadIdx.x;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CH;
    const int ch = lane / LPC;   // channel within the warp
    const int sub = lane % LPC;  // which SPL states
    const int d = d0 + ch;
    const bool active = d < D;
    const size_t row0 = (size_t)b * L;

    int32_t h[SPL], nn[SPL];
    int bad = 0;
    const int32_t lim = 1 << k;
#pragma unroll
    for (int j = 0; j < SPL; j++) {
        const int jj = sub * SPL + j;
        h[j] = active ? h_io[((size_t)b * D + d) * NS + jj] : 0;
        nn[j] = active ? n[(size_t)d * NS + jj] : 0;
        bad |= (nn[j] < 0) | (nn[j] > lim);
    }

    int ovf = 0;  // sign-test accumulator: negative => an int32 state or y32 overflowed
    const int nchunks = cdiv(L, TC);
#pragma unroll
    for (int c = 0; c < SST - 1; c++) {
        if (c < nchunks) load_chunk<CH>(stage[c], c * TC, x, Bm, Cm, row0, d0, L, D);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    for (int c = 0; c < nchunks; c++) {
        Stage<CH>& st = stage[c % SST];
        // the slot refilled here was emptied by the previous iteration
        if (c + SST - 1 < nchunks)
            load_chunk<CH>(stage[(c + SST - 1) % SST], (c + SST - 1) * TC, x, Bm, Cm, row0, d0, L, D);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group %0;\n" ::"n"(SST - 1) : "memory");
        __syncwarp();
        // range check of the staged inputs
#pragma unroll
        for (int i = lane; i < TC * CH / 4; i += 32) bad |= out_of_range4(reinterpret_cast<const int4*>(&st.x[0][0])[i]);
#pragma unroll
        for (int i = lane; i < TC * 2 * NS / 4; i += 32)
            bad |= out_of_range4(reinterpret_cast<const int4*>(&st.bc[0][0])[i]);
        const int t0 = c * TC;
        const int tn = min(TC, L - t0);
#pragma unroll 2
        for (int r = 0; r < tn; r++) {
            const int32_t xv = st.x[r][ch];
            int32_t bb[SPL], cc[SPL];
#pragma unroll
            for (int q = 0; q < SPL / 4; q++) {
                const int4 b4 = *reinterpret_cast<const int4*>(&st.bc[r][sub * SPL + 4 * q]);
                const int4 c4 = *reinterpret_cast<const int4*>(&st.bc[r][NS + sub * SPL + 4 * q]);
                bb[4 * q] = b4.x; bb[4 * q + 1] = b4.y; bb[4 * q + 2] = b4.z; bb[4 * q + 3] = b4.w;
                cc[4 * q] = c4.x; cc[4 * q + 1] = c4.y; cc[4 * q + 2] = c4.z; cc[4 * q + 3] = c4.w;
            }
            // two independent 64-bit multiply-add chains for y (integer sums are
            // exact in any order)
            long long acc0 = 0, acc1 = 0;
            int32_t ovl = 0;
#pragma unroll
            for (int j = 0; j < SPL; j++) {
                const long long p = (long long)h[j] * (long long)nn[j];
                const int32_t s = (int32_t)(p >> k);
                const int32_t bx = (int32_t)((uint32_t)bb[j] * (uint32_t)xv);  // |B*x| < 2^30 when in range
                const int32_t hn = (int32_t)((uint32_t)s + (uint32_t)bx);
                ovl |= (s ^ hn) & (bx ^ hn);
                h[j] = hn;
                if (j & 1) acc1 += (long long)cc[j] * (long long)hn;
                else acc0 += (long long)cc[j] * (long long)hn;
            }
            ovf |= ovl;
            long long acc = acc0 + acc1;
#pragma unroll
            for (int o = 1; o < LPC; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (sub == 0) ys[r][ch] = acc;
        }
        __syncwarp();
        // write the chunk's y rows: TC rows x CH values as 16-byte vectors
        if (Y64) {
#pragma unroll
            for (int i = lane; i < TC * (CH / 2); i += 32) {
                const int r = i / (CH / 2), q = i % (CH / 2);  // chunks of two int64 per row
                const int dq = d0 + 2 * q;
                if (r < tn && dq < D) {
                    int64_t* o = y64 + (row0 + t0 + r) * D + dq;
                    *reinterpret_cast<longlong2*>(o) = make_longlong2(ys[r][2 * q], ys[r][2 * q + 1]);
                }
            }
        } else {
#pragma unroll
            for (int i = lane; i < TC * (CH / 4); i += 32) {
                const int r = i / (CH / 4), q = i % (CH / 4);  // chunks of four int32 per row
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
        __syncwarp();  // ys and the stage slot are rewritten in the next iterations
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");

    if (active) {
        int4* hp = reinterpret_cast<int4*>(h_io + ((size_t)b * D + d) * NS + sub * SPL);
#pragma unroll
        for (int q = 0; q < SPL / 4; q++) hp[q] = make_int4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
    }
    if (ovf < 0) raise_dev_error(MI_DEV_OVERFLOW);
    if (bad) raise_dev_error(MI_DEV_PRECOND);
}

template <int LPC>
static void launch_scan_i32(const int32_t* x, const int32_t* B, const int32_t* C, const int32_t* n, int k,
                            int32_t* y32, int64_t* y64, int32_t* h_io, int batch, int L, int D, cudaStream_t s) {
    dim3 grid(cdiv(D, Geo<LPC>::CH), batch);
    if (y64)
        scan_i32_kernel<LPC, true><<<grid, THREADS, 0, s>>>(x, B, C, n, k, nullptr, y64, h_io, L, D);
    else
        scan_i32_kernel<LPC, false><<<grid, THREADS, 0, s>>>(x, B, C, n, k, y32, nullptr, h_io, L, D);
}

}  // namespace scan_i32
}  // namespace mi

extern "C" int mi_scan_i32(const int32_t* x, const int32_t* B, const int32_t* C, const int32_t* n, int k,
                           int32_t* y32, int64_t* y64, int32_t* h_io, int batch, int L, int D, int N,
                           void* stream) {
    using namespace mi::scan_i32;
    using mi::cdiv;
    if (!x || !B || !C || !n || !h_io) return MI_ERR_INVALID;
    if ((y32 == nullptr) == (y64 == nullptr)) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || D <= 0) return MI_ERR_INVALID;
    if (N != NS) return MI_ERR_UNSUPPORTED;
    if (k < 1 || k > 30) return MI_ERR_UNSUPPORTED;
    if (D % 4 != 0) return MI_ERR_UNSUPPORTED;  // 16-byte staging of x rows and vector y stores
    if (((uintptr_t)x | (uintptr_t)B | (uintptr_t)C | (uintptr_t)y32 | (uintptr_t)y64 | (uintptr_t)h_io) & 15)
        return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    // 2 lanes per channel; 4 when the batch leaves too few warps to fill the GPU
    if ((long long)batch * cdiv(D, Geo<2>::CH) >= 4LL * 148)
        launch_scan_i32<2>(x, B, C, n, k, y32, y64, h_io, batch, L, D, s);
    else
        launch_scan_i32<4>(x, B, C, n, k, y32, y64, h_io, batch, L, D, s);
    MI_CHECK_LAUNCH();
    return MI_OK;
}
