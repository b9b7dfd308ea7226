// scan_i32.cu -- integer dyadic selective scan (sm_100a).
//
//   h[b,d,j] <- ((int64)h * n[d,j]) >> k  +  B[b,t,j] * x[b,t,d]
//   y[b,t,d]  = sum_j C[b,t,j] * h[b,d,j]
//
// The state update follows the reference POC kernel
// (src/cuda_kernels/dyadic_mamba_kernel.cu:53-59: 64-bit product, arithmetic
// right shift, add) with the selective-scan input term B_t*x_t and the output
// contraction C_t.h_t added.  The shifted product is formed as the high word
// of a 32-bit multiply (see scan_step), which gives the same integer.
//
// Layout / parallelism: one warp per CTA owns 32/LPC channels of one
// sequence; LPC lanes per channel each hold 16/LPC of the 16 int32 states in
// registers for the whole sequence (the recurrence is sequential in t, so the
// independent (sequence, channel, state) chains are all the parallelism there
// is).  x and B|C arrive through a per-warp 4-deep cp.async ring of TC-step
// chunks (three chunks in flight ahead of the one in use, no block-level
// barriers).  A full chunk runs as one unrolled block, so that the loads and
// y sums of a step overlap the state chains of the next ones (the kernel is
// bound by dependency latency: few warps per SM, each a serial recurrence).
// The LPC partial y sums of a channel meet in shuffles and each step's y
// row segment (CH consecutive channels) is stored at once, with no staging.
// LPC = 2 at config 2 sizes: the B|C values every lane must receive each
// step share the load/store data path, which fewer lanes per channel use
// less of.
//
// Exactness: the shifted product fits int32 whenever 0 <= n <= 2^k, and its
// magnitude never exceeds |h|; |B*x| < 2^30 when |B|,|x| <= 32767.  Per chunk,
// the staged inputs' largest magnitudes and the warp's largest state bound
// every state and every y partial sum of the chunk; where that bound fits
// int32 the chunk runs with 32-bit arithmetic only, otherwise each state add
// is checked for int32 overflow with a sign test and y is summed in 64 bits.
// Violations set the device error word instead of producing wrong values
// silently.
#include <type_traits>

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

// One time step of one lane's SPL states.  The LPC partial y sums of a
// channel meet in shuffles and the channel's first lane stores y to `yout`
// (a warp stores CH consecutive values of the row in one instruction).
//
// The shifted product floor(h * n / 2^k) is the high word of h * (n * 2^(32-k)):
// with m = n << (32 - k) taken as a signed int32, mul.hi gives
// floor(h * m / 2^32), which is 2^32 * h too small exactly when n * 2^(32-k)
// >= 2^31 (m wrapped negative, or to 0 for n = 2^k), so the lane adds h there
// (am = -1 selects it).  0 <= n <= 2^k keeps |result| <= |h|.  AMALL: every
// n of the warp is >= 2^(k-1), so h is added back unconditionally (the add
// folds into the multiply-high).
//
// FAST: the chunk's bound (checked by the caller) rules out every int32
// overflow of the states and of 32-bit y sums, so neither is tested or
// widened.  Otherwise the y sums are 64-bit and each state add is checked.
template <int LPC, bool FAST, bool AMALL, typename Out>
__device__ __forceinline__ void scan_step(int32_t (&h)[Geo<LPC>::SPL], const int32_t (&nm)[Geo<LPC>::SPL],
                                          const int32_t (&am)[Geo<LPC>::SPL], int32_t xv,
                                          const int32_t* __restrict__ bc_row, int sub, Out* __restrict__ yout,
                                          bool store, int32_t& ovf) {
    constexpr int SPL = Geo<LPC>::SPL;
    constexpr int NACC = SPL < 4 ? SPL : 4;  // independent multiply-add chains for y
    int32_t bb[SPL], cc[SPL];
#pragma unroll
    for (int q = 0; q < SPL / 4; q++) {
        const int4 b4 = *reinterpret_cast<const int4*>(&bc_row[sub * SPL + 4 * q]);
        const int4 c4 = *reinterpret_cast<const int4*>(&bc_row[NS + sub * SPL + 4 * q]);
        bb[4 * q] = b4.x; bb[4 * q + 1] = b4.y; bb[4 * q + 2] = b4.z; bb[4 * q + 3] = b4.w;
        cc[4 * q] = c4.x; cc[4 * q + 1] = c4.y; cc[4 * q + 2] = c4.z; cc[4 * q + 3] = c4.w;
    }
    // integer sums are exact in any order
    using Acc = typename std::conditional<FAST, int32_t, long long>::type;
    Acc acc[NACC];
#pragma unroll
    for (int a = 0; a < NACC; a++) acc[a] = 0;
    int32_t ovl = 0;
#pragma unroll
    for (int j = 0; j < SPL; j++) {
        const int32_t s = __mulhi(h[j], nm[j]) + (AMALL ? h[j] : (h[j] & am[j]));
        const int32_t bx = (int32_t)((uint32_t)bb[j] * (uint32_t)xv);  // |B*x| < 2^30 when in range
        const int32_t hn = (int32_t)((uint32_t)s + (uint32_t)bx);
        if (!FAST) ovl |= (s ^ hn) & (bx ^ hn);
        h[j] = hn;
        acc[j % NACC] += (Acc)cc[j] * (Acc)hn;
    }
    if (!FAST) ovf |= ovl;
#pragma unroll
    for (int w = NACC / 2; w >= 1; w /= 2)
#pragma unroll
        for (int a = 0; a < w; a++) acc[a] += acc[a + w];
    Acc y = acc[0];
#pragma unroll
    for (int o = 1; o < LPC; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
    if (store) {
        if (sizeof(Out) == 4 && !FAST && ((long long)y > INT32_MAX || (long long)y < INT32_MIN)) ovf |= INT32_MIN;
        *yout = (Out)y;
    }
}

__device__ __forceinline__ unsigned uabs(int32_t v) {
    const unsigned u = (unsigned)v;
    return v < 0 ? 0u - u : u;  // 2^31 for INT32_MIN
}
__device__ __forceinline__ unsigned absmax4(int4 v) {
    return max(max(uabs(v.x), uabs(v.y)), max(uabs(v.z), uabs(v.w)));
}

// The steps of one staged chunk (tn of them); y of step r goes to yb + r * D.
template <int LPC, bool FAST, bool AMALL, int CH, typename Out>
__device__ __forceinline__ void scan_chunk(int32_t (&h)[Geo<LPC>::SPL], const int32_t (&nm)[Geo<LPC>::SPL],
                                           const int32_t (&am)[Geo<LPC>::SPL], const Stage<CH>& st, Out* yb,
                                           int D, bool store, int tn, int ch, int sub, int32_t& ovf) {
    if (tn == TC) {
        // a full chunk as one straight-line block: the steps' loads, y sums and
        // stores overlap the state chains of the following steps
#pragma unroll
        for (int r = 0; r < TC; r++)
            scan_step<LPC, FAST, AMALL>(h, nm, am, st.x[r][ch], st.bc[r], sub, yb + (size_t)r * D, store, ovf);
    } else {
#pragma unroll 1
        for (int r = 0; r < tn; r++)
            scan_step<LPC, FAST, AMALL>(h, nm, am, st.x[r][ch], st.bc[r], sub, yb + (size_t)r * D, store, ovf);
    }
}

template <int LPC, bool Y64>
__global__ void __launch_bounds__(THREADS)
scan_i32_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ Bm, const int32_t* __restrict__ Cm,
                const int32_t* __restrict__ n, const int k, int32_t* __restrict__ y32, int64_t* __restrict__ y64,
                int32_t* __restrict__ h_io, int L, int D) {
    using G = Geo<LPC>;
    constexpr int SPL = G::SPL, CH = G::CH;
    __shared__ __align__(16) Stage<CH> stage[SST];
    const int lane = threadIdx.x;
    const int b = blockIdx.y;
    const int d0 = blockIdx.x * CH;
    const int ch = lane / LPC;   // channel within the warp
    const int sub = lane % LPC;  // which SPL states
    const int d = d0 + ch;
    const bool active = d < D;
    const bool store = active && sub == 0;
    const size_t row0 = (size_t)b * L;

    // states, and each n as the multiplier n << (32 - k) and the add-back mask
    int32_t h[SPL], nm[SPL], am[SPL];
    int bad = 0;
    const int32_t lim = 1 << k;
#pragma unroll
    for (int j = 0; j < SPL; j++) {
        const int jj = sub * SPL + j;
        h[j] = active ? h_io[((size_t)b * D + d) * NS + jj] : 0;
        const int32_t nv = active ? n[(size_t)d * NS + jj] : 0;
        bad |= (nv < 0) | (nv > lim);
        nm[j] = (int32_t)((uint32_t)nv << (32 - k));
        am[j] = (nv >= (lim >> 1)) ? -1 : 0;
    }
    int lane_amall = 1;
#pragma unroll
    for (int j = 0; j < SPL; j++) lane_amall &= (am[j] == -1);
    const bool amall = __all_sync(0xffffffffu, lane_amall);

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
        // the staged inputs' largest magnitudes (range check and chunk bound)
        unsigned mx = 0, mb = 0, mc = 0;
#pragma unroll
        for (int i = lane; i < TC * CH / 4; i += 32)
            mx = max(mx, absmax4(reinterpret_cast<const int4*>(&st.x[0][0])[i]));
#pragma unroll
        for (int i = lane; i < TC * 2 * NS / 4; i += 32) {  // 8 int4 per row: B in 0..3, C in 4..7
            const unsigned m = absmax4(reinterpret_cast<const int4*>(&st.bc[0][0])[i]);
            if ((i & 7) < 4) mb = max(mb, m);
            else mc = max(mc, m);
        }
        unsigned hm = 0;
#pragma unroll
        for (int j = 0; j < SPL; j++) hm = max(hm, uabs(h[j]));
        mx = __reduce_max_sync(0xffffffffu, mx);
        mb = __reduce_max_sync(0xffffffffu, mb);
        mc = __reduce_max_sync(0xffffffffu, mc);
        hm = __reduce_max_sync(0xffffffffu, hm);
        // |h| grows by at most |B*x| per step (|floor(h*n/2^k)| <= |h|), so over the
        // chunk every state stays within hb and every partial y sum within NS*|C|*hb
        bool fast = mx <= 32767u && mb <= 32767u && mc <= 32767u;
        bad |= !fast;  // |x|, |B| or |C| above 32767
        if (fast) {
            const unsigned long long hb = (unsigned long long)hm + (unsigned long long)TC * mb * mx;
            fast = hb <= (unsigned long long)INT32_MAX && (unsigned long long)NS * mc * hb <= (unsigned long long)INT32_MAX;
        }
        const int t0 = c * TC;
        const int tn = min(TC, L - t0);
        const size_t yoff = (row0 + t0) * D + (active ? d : 0);
        if (Y64) {
            if (fast && amall)
                scan_chunk<LPC, true, true, CH>(h, nm, am, st, y64 + yoff, D, store, tn, ch, sub, ovf);
            else if (fast)
                scan_chunk<LPC, true, false, CH>(h, nm, am, st, y64 + yoff, D, store, tn, ch, sub, ovf);
            else
                scan_chunk<LPC, false, false, CH>(h, nm, am, st, y64 + yoff, D, store, tn, ch, sub, ovf);
        } else {
            if (fast && amall)
                scan_chunk<LPC, true, true, CH>(h, nm, am, st, y32 + yoff, D, store, tn, ch, sub, ovf);
            else if (fast)
                scan_chunk<LPC, true, false, CH>(h, nm, am, st, y32 + yoff, D, store, tn, ch, sub, ovf);
            else
                scan_chunk<LPC, false, false, CH>(h, nm, am, st, y32 + yoff, D, store, tn, ch, sub, ovf);
        }
        __syncwarp();  // the stage slot is refilled by the next iteration
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
