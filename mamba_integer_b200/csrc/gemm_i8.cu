// gemm_i8.cu -- ternary BitLinear contraction on the 5th-generation tensor
// cores: C[m,n] = sum_k A[m,k] * W[n,k] with A the int8 activations and W the
// ternary weights stored as int8, tcgen05.mma kind::i8 with int32
// accumulators in tensor memory.
//
// Persistent, one CTA per SM, BM x BN output tiles (BM = 128 rows of tokens):
//   warp 0 / lane 0  TMA producer: 2-D tiled loads (128-byte swizzle) of the
//                    A and W K-slices into a STAGES-deep shared-memory ring;
//   warp 1 / lane 0  MMA issuer: 4 x tcgen05.mma (K = 32 bytes each) per
//                    128-byte K-slice into one of two TMEM accumulators,
//                    tcgen05.commit frees the ring slot / hands the
//                    accumulator to the epilogue;
//   warps 2-5        epilogue: tcgen05.ld 32x32b (one accumulator row per
//                    thread), dequantise acc * (w_scale * a_scale[m])
//                    [* out_scale] exactly as BitLinear.forward does
//                    (src/rational_bitnet.py:204-208), stage 32x32 boxes in
//                    swizzled shared memory, TMA bulk tensor store;
//   warps 6-13       (2-bit packed weights only) unpack: the TMA brings the
//                    K-slice of packed weights (BN rows x 32 bytes); these
//                    warps expand it to int8 in the 128-byte-swizzled layout
//                    the MMA reads, then release the stage to the MMA issuer.
// Every mbarrier wait is bounded (about 2 s of clock); on expiry the CTA sets
// MI_DEV_TIMEOUT, stops issuing, frees its tensor memory and exits.
//
// The accumulation is exact: |sum| <= 127*K < 2^31, and int -> fp32 is exact
// below 2^24 (K <= 132104), the range every BitLinear of the model is in.
#include <cstdlib>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "mi_common.cuh"

namespace mi {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes (= int8 elements) of K per stage: one 128-byte swizzle row
constexpr int BKP = BK / 4;  // bytes of one packed K-slice row (4 ternary weights per byte)
constexpr int EPI_WARPS = 4;
constexpr int UNPACK_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;  // producer warp, MMA warp, 4 epilogue warps
constexpr int THREADS_PACKED = THREADS + 32 * UNPACK_WARPS;  // + 8 unpack warps
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s at 2 GHz

template <bool PACKED>
constexpr int threads_of() { return PACKED ? THREADS_PACKED : THREADS; }

// HEAVY (packed 256-wide tiles over K >= 1536, where the tensor cores rather than
// the output stores set the pace): 12 unpack warps, a 6-slice load ring and one
// staging box per epilogue warp.  Config 3 (K 2048): 0.2416 against 0.2568 ms;
// the same setting on the store-bound K = 768 in_proj cost 0.24 ms per step.
template <int BN, bool PACKED = false, bool HEAVY = false>
struct Cfg {
    static constexpr bool H = PACKED && HEAVY && BN > 128;
    static constexpr int UW = H ? 12 : UNPACK_WARPS;                 // unpack warps (packed only)
    static constexpr int NTHREADS = THREADS + (PACKED ? 32 * UW : 0);
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int P_LOAD = PACKED ? BN * BKP : 0;             // packed bytes the TMA brings per stage
    static constexpr int P_BYTES = (P_LOAD + 1023) / 1024 * 1024;    // their slot, padded to the 1 KB pitch
    // Load ring: each stage holds the A slice and the weight slice (int8, or
    // packed).  Packed weights are expanded into a separate, shorter ring of
    // int8 tiles, so the load ring (small packed slices) can run deeper and
    // cover the load latency plus the unpack.  256-wide tiles read each A
    // slice once per 256 output columns.
    static constexpr int STAGES = PACKED ? (BN > 128 ? (H ? 6 : 5) : 6) : 4;
    static constexpr int STAGE_BYTES = A_BYTES + (PACKED ? P_BYTES : B_BYTES);
    static constexpr int BSTAGES = PACKED ? (BN > 128 ? 2 : 3) : 0;  // int8 weight tiles (packed only)
    static constexpr int BSM = BSTAGES > 0 ? BSTAGES : 1;           // modulus for the ring index
    static constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;  // per accumulator
    static constexpr int EPI_BOXES = (BN + 31) / 32;   // 32-column output boxes per tile
    static constexpr int STG_BUFS = H ? 1 : ((PACKED || BN > 128) ? 2 : 4);  // staging boxes per epilogue warp
    static constexpr int STG_BYTES = EPI_WARPS * STG_BUFS * 4096;  // (bulk stores kept in flight)
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BSTAGES * B_BYTES + STG_BYTES + BAR_BYTES;
    static_assert(B_BYTES % 1024 == 0, "int8 weight tiles keep the 1 KB alignment");
    static_assert(8 * (2 * STAGES + 4 + 2 * BSTAGES) + 8 <= BAR_BYTES, "barrier block");
    static_assert(STAGE_BYTES % 1024 == 0, "stage must keep 1024-byte alignment for the 128B swizzle");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
    static_assert(2 * TMEM_COLS <= 512, "two accumulators must fit in TMEM");
    static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: true when the phase completed, false on timeout / abort.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > WAIT_CYCLES) {
            *abort = 1;
            raise_dev_error(MI_DEV_TIMEOUT);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(
            dst),
        "l"((uint64_t)tm), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"((uint64_t)tm),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the canonical 128-byte
// swizzle layout written by TMA (8-row x 128-byte atoms, atoms 1024 B apart).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address  [0,14)
    d |= (uint64_t)1 << 16;                    // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: 8-row group pitch [32,46)
    d |= (uint64_t)1 << 46;                    // descriptor version for sm_100 [46,48)
    d |= (uint64_t)2 << 61;                    // layout: SWIZZLE_128B [61,64)
    return d;
}

// Instruction descriptor: kind::i8, D = s32, A/B signed int8, both K-major.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_i8() {
    return (2u << 4)                        // D format: S32
           | (1u << 7)                      // A format: signed 8-bit
           | (1u << 10)                     // B format: signed 8-bit
           | ((uint32_t)(BN >> 3) << 17)    // N / 8
           | ((uint32_t)(BM >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// ---------------------------------------------------------------------------
// 2-bit packed ternary weights.  Row n of the packed matrix holds K/4 bytes;
// each little-endian 32-bit word covers 16 consecutive weights k = 16g .. 16g+15,
// weight 16g + 4q + j in bits [p, p + 2), p = 4j + 2(q & 1) + 16(q >> 1), as a
// 2-bit two's complement value (00 = 0, 01 = +1, 11 = -1).  The layout puts
// the four codes of output word q in the low bits of the four nibbles of
// (w >> (2(q & 1) + 16(q >> 1))) & 0x3333, a byte-permute selector: one
// shift, one mask and one PRMT from the table {0, +1, 0, -1} per 4 weights.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t prmt_table(uint32_t sel) {
    uint32_t r;
    // source bytes 0..3 = 0x00, 0x01, 0x00, 0xFF (code 2 is never written)
    asm("prmt.b32 %0, %1, %1, %2;" : "=r"(r) : "r"(0xFF000100u), "r"(sel));
    return r;
}
__device__ __forceinline__ uint4 unpack16(uint32_t w) {
    return make_uint4(prmt_table(w & 0x3333u), prmt_table((w >> 2) & 0x3333u), prmt_table((w >> 16) & 0x3333u),
                      prmt_table((w >> 18) & 0x3333u));
}

// Expand one stage's packed K-slice (ROWS x 32 bytes, dense) into the int8
// tile (ROWS x 128 bytes, 128-byte swizzle: 16-byte chunk c of row r at
// c ^ (r & 7); the tile is 1024-byte aligned).  Each unpack thread takes
// 16-byte quads of packed bytes (4 words = 4 output chunks of one row), all
// loads issued before the stores; `tid` counts the unpack threads.
template <int ROWS, int UW = UNPACK_WARPS>
__device__ __forceinline__ void unpack_slice(const unsigned char* packed, unsigned char* tile, int tid) {
    constexpr int QUADS = ROWS * 2;  // a packed row is 2 quads
    constexpr int NT = 32 * UW;
    constexpr int ITERS = (QUADS + NT - 1) / NT;
    uint4 v[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; i++) {
        const int qd = tid + i * NT;
        if (qd < QUADS) v[i] = reinterpret_cast<const uint4*>(packed)[qd];
    }
#pragma unroll
    for (int i = 0; i < ITERS; i++) {
        const int qd = tid + i * NT;
        if (qd < QUADS) {
            const int r = qd >> 1, c0 = (qd & 1) * 4, sw = r & 7;
            unsigned char* row = tile + r * 128;
            *reinterpret_cast<uint4*>(row + (((c0 + 0) ^ sw) << 4)) = unpack16(v[i].x);
            *reinterpret_cast<uint4*>(row + (((c0 + 1) ^ sw) << 4)) = unpack16(v[i].y);
            *reinterpret_cast<uint4*>(row + (((c0 + 2) ^ sw) << 4)) = unpack16(v[i].z);
            *reinterpret_cast<uint4*>(row + (((c0 + 3) ^ sw) << 4)) = unpack16(v[i].w);
        }
    }
    // the MMA reads the tile through the async proxy
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Persistent kernel: each CTA walks the output tiles blockIdx.x,
// blockIdx.x + gridDim.x, ... (N fastest, so CTAs working at the same time
// share the A row-block in L2).  The smem ring and the two TMEM accumulators
// carry across tiles, so the epilogue of tile i overlaps the mainloop of
// tile i+1.
template <int BN, bool PACKED, bool HEAVY = false>
__global__ void __launch_bounds__(Cfg<BN, PACKED, HEAVY>::NTHREADS, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const float* __restrict__ a_scale,
               const float* __restrict__ w_scale, const float* __restrict__ out_scale, int M, int N, int K, int epi,
               unsigned long long* __restrict__ row_stats) {
    using C = Cfg<BN, PACKED, HEAVY>;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-aligned tiles
    unsigned char* gbase = smem_raw + (base - raw);
    const uint32_t wring = base + C::STAGES * C::STAGE_BYTES;       // int8 weight tiles (packed only)
    const uint32_t stg_base = wring + C::BSTAGES * C::B_BYTES;      // epilogue staging (1024-aligned)
    const uint32_t bars = stg_base + C::STG_BYTES;
    // barriers: full[S], empty[S], tfull[2], tempty[2], then (packed only)
    // bready[BS] (int8 tile written) and bfree[BS] (its MMAs done); then the
    // TMEM slot and the abort flag
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
    auto tfull_bar = [&](int a) { return bars + 8u * (2 * C::STAGES + a); };
    auto tempty_bar = [&](int a) { return bars + 8u * (2 * C::STAGES + 2 + a); };
    auto bready_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + 4 + b); };
    auto bfree_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + 4 + C::BSTAGES + b); };
    uint32_t* tmem_slot =
        reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (2 * C::STAGES + 4 + 2 * C::BSTAGES));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_k = cdiv(K, BK);
    const int tiles_n = cdiv(N, BN);
    const int num_tiles = cdiv(M, BM) * tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), EPI_WARPS);
        }
        for (int b = 0; b < C::BSTAGES; b++) {
            mbar_init(bready_bar(b), C::UW);
            mbar_init(bfree_bar(b), 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // the previous kernel's outputs (A, the scales) are complete and its TMEM is
    // free before this CTA allocates TMEM or loads anything
    grid_dependency_sync();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)(2 * C::TMEM_COLS))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int g = 0;  // global k-stage counter across tiles
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const int m0 = (tile / tiles_n) * BM;
                const int n0 = (tile % tiles_n) * BN;
                for (int i = 0; i < num_k; i++, g++) {
                    const int s = g % C::STAGES;
                    if (g >= C::STAGES && !mbar_wait(empty_bar(s), ((g / C::STAGES) - 1) & 1, abort_flag)) break;
                    const uint32_t sa = base + s * C::STAGE_BYTES;
                    if (PACKED) {
                        mbar_expect_tx(full_bar(s), C::A_BYTES + C::P_LOAD);
                        tma_load_2d(sa, &tmA, full_bar(s), i * BK, m0);
                        tma_load_2d(sa + C::A_BYTES, &tmB, full_bar(s), i * BKP, n0);
                    } else {
                        mbar_expect_tx(full_bar(s), C::A_BYTES + C::B_BYTES);
                        tma_load_2d(sa, &tmA, full_bar(s), i * BK, m0);
                        tma_load_2d(sa + C::A_BYTES, &tmB, full_bar(s), i * BK, n0);
                    }
                }
            }
            if (*abort_flag) {
                // let the loads already issued land before the CTA exits (bounded)
                for (int j = (g > C::STAGES ? g - C::STAGES : 0); j < g; j++) {
                    const long long t0 = clock64();
                    while (!mbar_try(full_bar(j % C::STAGES), (j / C::STAGES) & 1) && clock64() - t0 < WAIT_CYCLES) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_i8<BN>();
            int g = 0;
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, it++) {
                const int a = it & 1;
                if (it >= 2 && !mbar_wait(tempty_bar(a), ((it >> 1) - 1) & 1, abort_flag)) break;
                tc_fence_after();
                const uint32_t tacc = tmem + (uint32_t)(a * C::TMEM_COLS);
                bool ok = true;
                for (int i = 0; i < num_k; i++, g++) {
                    const int s = g % C::STAGES;
                    const int b = g % C::BSM;
                    if (!mbar_wait(full_bar(s), (g / C::STAGES) & 1, abort_flag) ||
                        (PACKED && !mbar_wait(bready_bar(b), (g / C::BSM) & 1, abort_flag))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base + s * C::STAGE_BYTES;
                    const uint32_t sb = PACKED ? wring + b * C::B_BYTES : sa + C::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; kk++) {
                        const uint64_t ad = sdesc_sw128(sa + kk * 32);
                        const uint64_t bd = sdesc_sw128(sb + kk * 32);
                        mma_i8(tacc, ad, bd, idesc, (i | kk) != 0);
                    }
                    mma_commit(empty_bar(s));
                    if (PACKED) mma_commit(bfree_bar(b));
                }
                if (!ok) break;
                mma_commit(tfull_bar(a));
            }
        }
    } else if (PACKED && warp >= 2 + EPI_WARPS) {
        // ---------------- unpack (warps 6 .. 6 + UW - 1) ----------------
        // Stage g: the packed slice of load slot g % STAGES is expanded into
        // int8 tile g % BSTAGES once that tile's previous MMAs completed.  The
        // load slot itself is released by the MMA commit (which follows this
        // stage's bready), so the packed bytes stay put while they are read.
        const int tid = threadIdx.x - 32 * (2 + EPI_WARPS);
        int g = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
            for (int i = 0; i < num_k; i++, g++) {
                const int s = g % C::STAGES;
                const int b = g % C::BSM;
                const bool ready = mbar_wait(full_bar(s), (g / C::STAGES) & 1, abort_flag) &&
                                   (g < C::BSTAGES || mbar_wait(bfree_bar(b), ((g / C::BSM) - 1) & 1, abort_flag));
                if (!__all_sync(0xffffffffu, ready)) {
                    ok = false;
                    break;
                }
                unpack_slice<BN, C::UW>(gbase + s * C::STAGE_BYTES + C::A_BYTES,
                                        gbase + (wring - base) + b * C::B_BYTES, tid);
                __syncwarp();
                if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bready_bar(b)) : "memory");
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        // A warp may only touch the TMEM lane quarter warp % 4: it owns the tile
        // rows q*32 .. q*32+31.  Each 32-column slab is dequantised, written in
        // the 128-byte-swizzled layout of a 32x32 TMA box into one of STG_BUFS
        // staging buffers, and stored with a bulk tensor copy (TMA clips rows
        // >= M and columns >= N); up to STG_BUFS stores stay in flight per warp.
        const int q = warp & 3;
        const uint32_t stg = stg_base + (uint32_t)((warp - 2) * C::STG_BUFS * 4096);
        unsigned char* stg_g = gbase + (stg - base);
        const float ws = (epi == MI_EPI_F32_SCALED) ? *w_scale : 0.0f;
        const float os = out_scale ? *out_scale : 1.0f;
        int it = 0, nst = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, it++) {
            const int a = it & 1;
            const bool have = __all_sync(0xffffffffu, mbar_wait(tfull_bar(a), (it >> 1) & 1, abort_flag));
            if (!have) break;
            tc_fence_after();
            const int m0 = (tile / tiles_n) * BM;
            const int n0 = (tile % tiles_n) * BN;
            const int row = m0 + q * 32 + lane;
            float sc = 0.0f;
            if (epi == MI_EPI_F32_SCALED && row < M) sc = __fmul_rn(ws, a_scale[row]);  // (w_scale * x_scale)
            const uint32_t tacc = tmem + (uint32_t)(a * C::TMEM_COLS) + ((uint32_t)(q * 32) << 16);
            long long s1 = 0, s2 = 0;  // exact row sums of this tile's accumulators (row_stats)
#pragma unroll 1
            for (int cb = 0; cb < C::EPI_BOXES; cb++, nst++) {
                uint32_t r[32] = {};
                tmem_ld16(tacc + (uint32_t)(cb * 32), *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
                if (cb * 32 + 16 < BN)
                    tmem_ld16(tacc + (uint32_t)(cb * 32 + 16), *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
                if (cb == C::EPI_BOXES - 1) {
                    // every TMEM read of this accumulator is done: hand it back to the MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(tempty_bar(a)) : "memory");
                }
                if (row_stats) {
                    // columns past N hold 0 (their weight rows were filled with zeros by the TMA)
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const long long v = (int32_t)r[j];
                        s1 += v;
                        s2 += v * v;
                    }
                }
                if (epi == MI_EPI_F32_SCALED) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        float v = __fmul_rn((float)(int32_t)r[j], sc);
                        if (out_scale) v = __fmul_rn(v, os);
                        r[j] = __float_as_uint(v);
                    }
                }
                // the staging buffer used STG_BUFS stores ago must have been read
                static_assert(C::STG_BUFS == 4 || C::STG_BUFS == 2 || C::STG_BUFS == 1, "power-of-two staging ring");
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(C::STG_BUFS - 1) : "memory");
                __syncwarp();
                unsigned char* rowp = stg_g + (nst & (C::STG_BUFS - 1)) * 4096 + lane * 128;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const int phys = c ^ (lane & 7);
                    *reinterpret_cast<uint4*>(rowp + phys * 16) =
                        make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    const int x = n0 + cb * 32, y = m0 + q * 32;
                    if (x < N && y < M) tma_store_2d(&tmC, stg + (nst & (C::STG_BUFS - 1)) * 4096, x, y);
                    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
                }
            }
            if (row_stats && row < M) {
                // two's complement: the unsigned 64-bit adds accumulate signed sums exactly
                atomicAdd(row_stats + 2 * (size_t)row, (unsigned long long)s1);
                atomicAdd(row_stats + 2 * (size_t)row + 1, (unsigned long long)s2);
            }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"((uint32_t)(2 * C::TMEM_COLS))
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// A-resident variant for K <= 768 (in_proj, lm_head): the 128-row block of A
// (up to 6 K-slices, 96 KB) is loaded once per work unit and kept in shared
// memory while the unit's N tiles stream their weight slices through a
// 6-deep ring, so A crosses L2 once per unit instead of once per N tile and
// the ring holds twice the bytes in flight of the streaming kernel.
// A unit is (M tile, group of consecutive N tiles); units go round-robin to
// the persistent CTAs.
// ---------------------------------------------------------------------------
constexpr int ARES_MAXK = 6;    // K slices held (K <= 768)
constexpr int ARES_BN = 128;
constexpr int ARES_STG = 2;     // staging boxes per epilogue warp
constexpr int ARES_A_BYTES = ARES_MAXK * BM * BK;              // 96 KB
constexpr int ARES_B_BYTES = ARES_BN * BK;                     // 16 KB per slice
constexpr int ARES_P_BYTES = ARES_BN * BKP;                    // 4 KB per packed slice
constexpr int ARES_STG_BYTES = EPI_WARPS * ARES_STG * 4096;    // 32 KB

// Weight rings: 6 int8 slices loaded by the TMA; or, with packed weights, 8
// packed slices in flight (TMA) feeding 3 int8 slices (written by the unpack
// warps, read by the MMAs).
template <bool PACKED>
struct AresCfg {
    static constexpr int SB = PACKED ? 3 : 6;
    static constexpr int PSB = PACKED ? 8 : 0;
    static constexpr int PSM = PSB > 0 ? PSB : 1;  // modulus for the packed ring index
    static constexpr int SMEM = 1024 + ARES_A_BYTES + SB * ARES_B_BYTES + PSB * ARES_P_BYTES + ARES_STG_BYTES + 256;
    static_assert(ARES_P_BYTES % 1024 == 0, "packed slices keep the 1 KB pitch");
    static_assert(8 * (2 * SB + 6 + 2 * PSB) + 8 <= 256, "barrier block");
    static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

template <bool PACKED>
__global__ void __launch_bounds__(threads_of<PACKED>(), 1)
gemm_i8_ares_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const float* __restrict__ a_scale,
                    const float* __restrict__ w_scale, const float* __restrict__ out_scale, int M, int N, int K,
                    int epi, int groups) {
    constexpr int BN = ARES_BN;
    constexpr int TMEM_COLS = 128;
    constexpr int EPI_BOXES = BN / 32;
    constexpr int ARES_SB = AresCfg<PACKED>::SB;
    constexpr int PSB = AresCfg<PACKED>::PSB;
    constexpr int PSM = AresCfg<PACKED>::PSM;
    constexpr int SLOT = ARES_B_BYTES;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (base - raw);
    const uint32_t a_base = base;                                   // ARES_MAXK x 16 KB
    const uint32_t b_base = a_base + ARES_A_BYTES;                  // ARES_SB int8 weight slices
    const uint32_t p_base = b_base + ARES_SB * SLOT;                // PSB packed slices (packed only)
    const uint32_t stg_base = p_base + PSB * ARES_P_BYTES;          // staging
    const uint32_t bars = stg_base + ARES_STG_BYTES;
    // barriers: bfull[SB] (int8 slice ready: TMA, or the unpack warps), bempty[SB]
    // (its MMAs done), tfull[2], tempty[2], afull, aempty, then (packed only)
    // pfull[PSB] (packed slice landed) and pempty[PSB] (unpacked); then TMEM
    // slot, abort flag
    auto bfull_bar = [&](int s) { return bars + 8u * s; };
    auto bempty_bar = [&](int s) { return bars + 8u * (ARES_SB + s); };
    auto tfull_bar = [&](int a) { return bars + 8u * (2 * ARES_SB + a); };
    auto tempty_bar = [&](int a) { return bars + 8u * (2 * ARES_SB + 2 + a); };
    const uint32_t afull_bar = bars + 8u * (2 * ARES_SB + 4);
    const uint32_t aempty_bar = bars + 8u * (2 * ARES_SB + 5);
    auto pfull_bar = [&](int s) { return bars + 8u * (2 * ARES_SB + 6 + s); };
    auto pempty_bar = [&](int s) { return bars + 8u * (2 * ARES_SB + 6 + PSB + s); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (2 * ARES_SB + 6 + 2 * PSB));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_k = cdiv(K, BK);
    const int tiles_n = cdiv(N, BN);
    const int tiles_m = cdiv(M, BM);
    const int units = tiles_m * groups;
    auto unit_range = [&](int u, int& m0, int& nt0, int& nt1) {
        const int g = u % groups;
        m0 = (u / groups) * BM;
        nt0 = (int)(((long long)g * tiles_n) / groups);
        nt1 = (int)(((long long)(g + 1) * tiles_n) / groups);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < ARES_SB; s++) {
            mbar_init(bfull_bar(s), PACKED ? UNPACK_WARPS : 1);
            mbar_init(bempty_bar(s), 1);
        }
        for (int s = 0; s < PSB; s++) {
            mbar_init(pfull_bar(s), 1);
            mbar_init(pempty_bar(s), UNPACK_WARPS);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), EPI_WARPS);
        }
        mbar_init(afull_bar, 1);
        mbar_init(aempty_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    grid_dependency_sync();  // as in gemm_i8_kernel
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)(2 * TMEM_COLS))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int g = 0, ua = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok && !*abort_flag; u += gridDim.x, ua++) {
                int m0, nt0, nt1;
                unit_range(u, m0, nt0, nt1);
                if (ua >= 1 && !mbar_wait(aempty_bar, (ua - 1) & 1, abort_flag)) break;
                mbar_expect_tx(afull_bar, (uint32_t)(num_k * BM * BK));
                for (int k = 0; k < num_k; k++) tma_load_2d(a_base + k * BM * BK, &tmA, afull_bar, k * BK, m0);
                for (int nt = nt0; nt < nt1 && ok; nt++) {
                    for (int k = 0; k < num_k; k++, g++) {
                        if (PACKED) {
                            const int s = g % PSM;
                            if (g >= PSB && !mbar_wait(pempty_bar(s), ((g / PSM) - 1) & 1, abort_flag)) {
                                ok = false;
                                break;
                            }
                            mbar_expect_tx(pfull_bar(s), (uint32_t)ARES_P_BYTES);
                            tma_load_2d(p_base + s * ARES_P_BYTES, &tmB, pfull_bar(s), k * BKP, nt * BN);
                        } else {
                            const int s = g % ARES_SB;
                            if (g >= ARES_SB && !mbar_wait(bempty_bar(s), ((g / ARES_SB) - 1) & 1, abort_flag)) {
                                ok = false;
                                break;
                            }
                            mbar_expect_tx(bfull_bar(s), (uint32_t)ARES_B_BYTES);
                            tma_load_2d(b_base + s * SLOT, &tmB, bfull_bar(s), k * BK, nt * BN);
                        }
                    }
                }
            }
            if (*abort_flag) {
                // let issued loads land before the CTA exits (bounded)
                const int ring = PACKED ? PSB : ARES_SB;
                for (int j = (g > ring ? g - ring : 0); j < g; j++) {
                    const long long t0 = clock64();
                    const uint32_t bar = PACKED ? pfull_bar(j % PSM) : bfull_bar(j % ARES_SB);
                    while (!mbar_try(bar, (j / ring) & 1) && clock64() - t0 < WAIT_CYCLES) {
                    }
                }
                if (ua > 0) {
                    const long long t0 = clock64();
                    while (!mbar_try(afull_bar, (ua - 1) & 1) && clock64() - t0 < WAIT_CYCLES) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_i8<BN>();
            int g = 0, it = 0, ua = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ua++) {
                int m0, nt0, nt1;
                unit_range(u, m0, nt0, nt1);
                if (!mbar_wait(afull_bar, ua & 1, abort_flag)) break;
                tc_fence_after();
                for (int nt = nt0; nt < nt1 && ok; nt++, it++) {
                    const int a = it & 1;
                    if (it >= 2 && !mbar_wait(tempty_bar(a), ((it >> 1) - 1) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t tacc = tmem + (uint32_t)(a * TMEM_COLS);
                    for (int k = 0; k < num_k; k++, g++) {
                        const int s = g % ARES_SB;
                        if (!mbar_wait(bfull_bar(s), (g / ARES_SB) & 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t sa = a_base + k * BM * BK;
                        const uint32_t sb = b_base + s * SLOT;
#pragma unroll
                        for (int kk = 0; kk < BK / 32; kk++)
                            mma_i8(tacc, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc, (k | kk) != 0);
                        mma_commit(bempty_bar(s));
                    }
                    if (!ok) break;
                    mma_commit(tfull_bar(a));
                }
                if (!ok) break;
                mma_commit(aempty_bar);  // the unit's MMAs have all read A once they complete
            }
        }
    } else if (PACKED && warp >= 2 + EPI_WARPS) {
        // ---------------- unpack (warps 6..13), as in gemm_i8_kernel ----------------
        const int tid = threadIdx.x - 32 * (2 + EPI_WARPS);
        int g = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            int m0, nt0, nt1;
            unit_range(u, m0, nt0, nt1);
            for (int nt = nt0; nt < nt1 && ok; nt++) {
                for (int k = 0; k < num_k; k++, g++) {
                    // packed slice g % PSB -> int8 slice g % SB (free once its MMAs completed)
                    const int ps = g % PSM, s = g % ARES_SB;
                    const bool ready = mbar_wait(pfull_bar(ps), (g / PSM) & 1, abort_flag) &&
                                       (g < ARES_SB || mbar_wait(bempty_bar(s), ((g / ARES_SB) - 1) & 1, abort_flag));
                    if (!__all_sync(0xffffffffu, ready)) {
                        ok = false;
                        break;
                    }
                    unpack_slice<BN>(gbase + (p_base - base) + ps * ARES_P_BYTES, gbase + (b_base - base) + s * SLOT,
                                     tid);
                    __syncwarp();
                    if (lane == 0) {
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(pempty_bar(ps)) : "memory");
                        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bfull_bar(s)) : "memory");
                    }
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5), as in gemm_i8_kernel ----------------
        const int q = warp & 3;
        const uint32_t stg = stg_base + (uint32_t)((warp - 2) * ARES_STG * 4096);
        unsigned char* stg_g = gbase + (stg - base);
        const float ws = (epi == MI_EPI_F32_SCALED) ? *w_scale : 0.0f;
        const float os = out_scale ? *out_scale : 1.0f;
        int it = 0, nst = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            int m0, nt0, nt1;
            unit_range(u, m0, nt0, nt1);
            const int row = m0 + q * 32 + lane;
            float sc = 0.0f;
            if (epi == MI_EPI_F32_SCALED && row < M) sc = __fmul_rn(ws, a_scale[row]);  // (w_scale * x_scale)
            for (int nt = nt0; nt < nt1; nt++, it++) {
                const int a = it & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(tfull_bar(a), (it >> 1) & 1, abort_flag))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int n0 = nt * BN;
                const uint32_t tacc = tmem + (uint32_t)(a * TMEM_COLS) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
                for (int cb = 0; cb < EPI_BOXES; cb++, nst++) {
                    uint32_t r[32];
                    tmem_ld16(tacc + (uint32_t)(cb * 32), *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
                    tmem_ld16(tacc + (uint32_t)(cb * 32 + 16), *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
                    if (cb == EPI_BOXES - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0)
                            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(tempty_bar(a)) : "memory");
                    }
                    if (epi == MI_EPI_F32_SCALED) {
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            float v = __fmul_rn((float)(int32_t)r[j], sc);
                            if (out_scale) v = __fmul_rn(v, os);
                            r[j] = __float_as_uint(v);
                        }
                    }
                    static_assert(ARES_STG == 2, "wait_group.read count below");
                    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory");
                    __syncwarp();
                    unsigned char* rowp = stg_g + (nst & (ARES_STG - 1)) * 4096 + lane * 128;
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const int phys = c ^ (lane & 7);
                        *reinterpret_cast<uint4*>(rowp + phys * 16) =
                            make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
                    }
                    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        const int x = n0 + cb * 32, y = m0 + q * 32;
                        if (x < N && y < M) tma_store_2d(&tmC, stg + (nst & (ARES_STG - 1)) * 4096, x, y);
                        asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
                    }
                }
            }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"((uint32_t)(2 * TMEM_COLS))
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D tensor [rows, cols] of `esize`-byte elements with row pitch ld_bytes;
// box = box_cols x box_rows, 128-byte swizzle (box_cols * esize == 128) or,
// with swizzle = false, a dense box (packed weight slices: 32-byte rows).
static int make_tmap(CUtensorMap* tm, const void* ptr, int rows, int cols, long long ld_bytes, int box_cols,
                     int box_rows, int esize, bool swizzle = true) {
    auto enc = get_encode();
    if (!enc) return MI_ERR_CUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUtensorMapDataType dt = esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    CUresult r = enc(tm, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MI_OK : MI_ERR_CUDA;
}

// Weight tensor map: int8 rows of K bytes (128-byte swizzled K-slices) or
// packed rows of K/4 bytes (dense 32-byte slices).
template <bool PACKED>
static int make_wmap(CUtensorMap* tm, const void* W, int N, int K, int box_rows) {
    if (PACKED) return make_tmap(tm, W, N, K / 4, K / 4, BKP, box_rows, 1, false);
    return make_tmap(tm, W, N, K, K, BK, box_rows, 1);
}

template <int BN, bool PACKED, bool HEAVY = false>
static int launch(const int8_t* A, int lda, const void* W, const float* a_scale, const float* w_scale,
                  const float* out_scale, void* out, int ldo, int M, int N, int K, int epi, cudaStream_t s,
                  unsigned long long* row_stats = nullptr) {
    // a tile whose last 32-column box sticks out past BN would overwrite the next tile
    if ((BN % 32) != 0 && N > BN) return MI_ERR_UNSUPPORTED;
    CUtensorMap ta, tb, tc;
    int rc = make_tmap(&ta, A, M, K, lda, BK, BM, 1);
    if (rc) return rc;
    rc = make_wmap<PACKED>(&tb, W, N, K, BN);
    if (rc) return rc;
    rc = make_tmap(&tc, out, M, N, (long long)ldo * 4, 32, 32, 4);
    if (rc) return rc;
    using C = Cfg<BN, PACKED, HEAVY>;
    if (cudaFuncSetAttribute(gemm_i8_kernel<BN, PACKED, HEAVY>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM) != cudaSuccess)
        return MI_ERR_CUDA;
    static int num_sms = 0;
    if (!num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (num_sms <= 0) num_sms = 148;
    }
    const int tiles = cdiv(M, BM) * cdiv(N, BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    MI_LAUNCH_DEPENDENT(gemm_i8_kernel<BN, PACKED, HEAVY>, dim3(grid), dim3(C::NTHREADS), C::SMEM, s, ta, tb, tc,
                        a_scale, w_scale, out_scale, M, N, K, epi, row_stats);
    return MI_OK;
}

static int sm_count() {
    static int num_sms = 0;
    if (!num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (num_sms <= 0) num_sms = 148;
    }
    return num_sms;
}

// ---------------------------------------------------------------------------
// 2-SM variant (tcgen05.mma.cta_group::2): a cluster of two CTAs computes one
// 256 x 256 output tile.  CTA rank r loads rows [m0 + 128r, +128) of A and the
// 128-row half [n0 + 128r, +128) of the weights into its own shared memory;
// the leader (rank 0) issues M=256, N=256 MMAs that read both CTAs' halves and
// accumulate rows 128r.. into CTA r's TMEM.  Per SM this halves the weight
// bytes staged and read per MMA, which is what bounds the one-CTA kernel
// (its shared-memory traffic per K-slice exceeds the MMA time).
// Synchronisation: the leader's full barrier counts both CTAs' TMA bytes
// (each CTA's loads signal it through its cluster address); MMA completions
// are committed to both CTAs' barriers (multicast commit); the epilogue warps
// of both CTAs arrive on the leader's barrier remotely.  No TMA multicast:
// each CTA loads its own operands.  All waits are bounded, and every path
// reaches the final cluster barrier before TMEM is freed.
// Int8 weights only: a packed-weight version (each CTA expanding its weight
// half, the peer's readiness relayed to the leader) was correct but slower
// than the one-CTA packed kernel at config 3 (0.38 vs 0.25 ms), so packed
// weights keep the one-CTA kernels.
// ---------------------------------------------------------------------------
constexpr int BM2 = 256;   // M of the pair's MMA (128 rows per CTA)
constexpr int BN2 = 256;   // N of the pair's MMA (128 weight rows per CTA)
constexpr int HALF = 128;

struct Cfg2 {
    static constexpr int A_BYTES = HALF * BK;   // this CTA's A rows
    static constexpr int B_BYTES = HALF * BK;   // this CTA's weight half
    // six stages and one staging box per epilogue warp measured best at config 3
    // (0.1885 ms, against 0.200 with five stages and two boxes)
    static constexpr int STAGES = 6;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 256;       // per accumulator (N = 256)
    static constexpr int EPI_BOXES = BN2 / 32;
    static constexpr int STG_BUFS = 1;
    static constexpr int STG_BYTES = EPI_WARPS * STG_BUFS * 4096;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + STG_BYTES + BAR_BYTES;
    static_assert(STAGE_BYTES % 1024 == 0, "1024-byte alignment of the swizzled tiles");
    static_assert(8 * (2 * STAGES + 4) + 16 <= BAR_BYTES, "barrier block");
    static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

__host__ __device__ constexpr uint32_t idesc_i8_2sm() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN2 >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose bytes complete on the pair leader's barrier
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* tm, uint32_t leader_bar, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];\n" ::"r"(dst),
        "l"((uint64_t)tm), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void mma_i8_2sm(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n}\n" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}
// completion of the issued MMAs arrives once on the barrier at this offset in both CTAs of the pair
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n" ::"r"(
            bar),
        "h"((uint16_t)3)
        : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
gemm2_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const float* __restrict__ a_scale,
                const float* __restrict__ w_scale, const float* __restrict__ out_scale, int M, int N, int K,
                int epi) {
    using C = Cfg2;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (base - raw);
    const uint32_t stg_base = base + C::STAGES * C::STAGE_BYTES;    // epilogue staging
    const uint32_t bars = stg_base + C::STG_BYTES;
    // barriers (same offsets in both CTAs): full[S] (leader: both CTAs' TMA bytes), empty[S],
    // tfull[2], tempty[2] (leader: 2 x EPI_WARPS arrivals)
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
    auto tfull_bar = [&](int a) { return bars + 8u * (2 * C::STAGES + a); };
    auto tempty_bar = [&](int a) { return bars + 8u * (2 * C::STAGES + 2 + a); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * (2 * C::STAGES + 4));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int num_k = cdiv(K, BK);
    const int tiles_n = cdiv(N, BN2);
    const int num_tiles = cdiv(M, BM2) * tiles_n;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 2 * EPI_WARPS);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)(2 * C::TMEM_COLS))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    // both CTAs' barriers are initialised and their TMEM allocated before either CTA
    // signals the other's barriers or the leader issues MMAs into it
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int g = 0;
            for (int tile = pair; tile < num_tiles && !*abort_flag; tile += npairs) {
                const int m0 = (tile / tiles_n) * BM2 + HALF * (int)rank;
                const int n0 = (tile % tiles_n) * BN2 + HALF * (int)rank;
                for (int i = 0; i < num_k; i++, g++) {
                    const int s = g % C::STAGES;
                    if (g >= C::STAGES && !mbar_wait(empty_bar(s), ((g / C::STAGES) - 1) & 1, abort_flag)) break;
                    const uint32_t sa = base + s * C::STAGE_BYTES;
                    const uint32_t lead_full = map_to_rank(full_bar(s), 0);
                    if (rank == 0) mbar_expect_tx(full_bar(s), 2 * (C::A_BYTES + C::B_BYTES));
                    tma_load_2d_pair(sa, &tmA, lead_full, i * BK, m0);
                    tma_load_2d_pair(sa + C::A_BYTES, &tmB, lead_full, i * BK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (the pair leader) ----------------
            constexpr uint32_t idesc = idesc_i8_2sm();
            int g = 0;
            int it = 0;
            for (int tile = pair; tile < num_tiles; tile += npairs, it++) {
                const int a = it & 1;
                if (it >= 2 && !mbar_wait(tempty_bar(a), ((it >> 1) - 1) & 1, abort_flag)) break;
                tc_fence_after();
                const uint32_t tacc = tmem + (uint32_t)(a * C::TMEM_COLS);
                bool ok = true;
                for (int i = 0; i < num_k; i++, g++) {
                    const int s = g % C::STAGES;
                    if (!mbar_wait(full_bar(s), (g / C::STAGES) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base + s * C::STAGE_BYTES;
                    const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 32; kk++)
                        mma_i8_2sm(tacc, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc, (i | kk) != 0);
                    mma_commit_pair(empty_bar(s));
                }
                if (!ok) break;
                mma_commit_pair(tfull_bar(a));
            }
        }
    } else if (warp >= 2 && warp < 2 + EPI_WARPS) {
        // ---------------- epilogue (both CTAs: each its 128 rows) ----------------
        const int q = warp & 3;
        const uint32_t stg = stg_base + (uint32_t)((warp - 2) * C::STG_BUFS * 4096);
        unsigned char* stg_g = gbase + (stg - base);
        const float ws = (epi == MI_EPI_F32_SCALED) ? *w_scale : 0.0f;
        const float os = out_scale ? *out_scale : 1.0f;
        int it = 0, nst = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs, it++) {
            const int a = it & 1;
            const bool have = __all_sync(0xffffffffu, mbar_wait(tfull_bar(a), (it >> 1) & 1, abort_flag));
            if (!have) break;
            tc_fence_after();
            const int m0 = (tile / tiles_n) * BM2 + HALF * (int)rank;
            const int n0 = (tile % tiles_n) * BN2;
            const int row = m0 + q * 32 + lane;
            float sc = 0.0f;
            if (epi == MI_EPI_F32_SCALED && row < M) sc = __fmul_rn(ws, a_scale[row]);
            const uint32_t tacc = tmem + (uint32_t)(a * C::TMEM_COLS) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
            for (int cb = 0; cb < C::EPI_BOXES; cb++, nst++) {
                uint32_t r[32];
                tmem_ld16(tacc + (uint32_t)(cb * 32), *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
                tmem_ld16(tacc + (uint32_t)(cb * 32 + 16), *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
                if (cb == C::EPI_BOXES - 1) {
                    // every TMEM read of this accumulator is done: tell the leader's MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(map_to_rank(tempty_bar(a), 0));
                }
                if (epi == MI_EPI_F32_SCALED) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        float v = __fmul_rn((float)(int32_t)r[j], sc);
                        if (out_scale) v = __fmul_rn(v, os);
                        r[j] = __float_as_uint(v);
                    }
                }
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(C::STG_BUFS - 1) : "memory");
                __syncwarp();
                unsigned char* rowp = stg_g + (nst & (C::STG_BUFS - 1)) * 4096 + lane * 128;
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const int phys = c ^ (lane & 7);
                    *reinterpret_cast<uint4*>(rowp + phys * 16) =
                        make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
                }
                asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    const int x = n0 + cb * 32, y = m0 + q * 32;
                    if (x < N && y < M) tma_store_2d(&tmC, stg + (nst & (C::STG_BUFS - 1)) * 4096, x, y);
                    asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
                }
            }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    // neither CTA frees TMEM or leaves while the other may still use the pair's resources
    cluster_sync_all();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"((uint32_t)(2 * C::TMEM_COLS))
                     : "memory");
    }
}

static int launch2(const int8_t* A, int lda, const void* W, const float* a_scale, const float* w_scale,
                   const float* out_scale, void* out, int ldo, int M, int N, int K, int epi, cudaStream_t s) {
    CUtensorMap ta, tb, tc;
    int rc = make_tmap(&ta, A, M, K, lda, BK, HALF, 1);
    if (rc) return rc;
    rc = make_wmap<false>(&tb, W, N, K, HALF);
    if (rc) return rc;
    rc = make_tmap(&tc, out, M, N, (long long)ldo * 4, 32, 32, 4);
    if (rc) return rc;
    using C = Cfg2;
    if (cudaFuncSetAttribute(gemm2_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess) {
        cudaGetLastError();
        return MI_ERR_CUDA;
    }
    // as many pairs as can be resident at once (a GPC with an odd number of free SMs
    // holds one pair fewer than half its SMs), so no pair waits for a second wave
    static int resident = 0;
    if (!resident) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
        cfg.blockDim = dim3(THREADS, 1, 1);
        cfg.dynamicSmemBytes = C::SMEM;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm2_i8_kernel, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = sm_count() / 2;
        }
        resident = n < sm_count() / 2 ? n : sm_count() / 2;
    }
    const int tiles = cdiv(M, BM2) * cdiv(N, BN2);
    int pairs = resident;
    if (pairs > tiles) pairs = tiles;
    gemm2_i8_kernel<<<2 * pairs, THREADS, C::SMEM, s>>>(ta, tb, tc, a_scale, w_scale, out_scale, M, N, K, epi);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

template <bool PACKED>
static int launch_ares(const int8_t* A, int lda, const void* W, const float* a_scale, const float* w_scale,
                       const float* out_scale, void* out, int ldo, int M, int N, int K, int epi, cudaStream_t s) {
    CUtensorMap ta, tb, tc;
    int rc = make_tmap(&ta, A, M, K, lda, BK, BM, 1);
    if (rc) return rc;
    rc = make_wmap<PACKED>(&tb, W, N, K, ARES_BN);
    if (rc) return rc;
    rc = make_tmap(&tc, out, M, N, (long long)ldo * 4, 32, 32, 4);
    if (rc) return rc;
    constexpr int SMEM = AresCfg<PACKED>::SMEM;
    if (cudaFuncSetAttribute(gemm_i8_ares_kernel<PACKED>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) !=
        cudaSuccess)
        return MI_ERR_CUDA;
    const int sms = sm_count();
    const int tiles_m = cdiv(M, BM), tiles_n = cdiv(N, ARES_BN);
    // split each M tile's N range into groups until there are >= 2 units per SM
    int groups = cdiv(2 * sms, tiles_m);
    if (groups < 1) groups = 1;
    if (groups > tiles_n) groups = tiles_n;
    const int units = tiles_m * groups;
    const int grid = units < sms ? units : sms;
    MI_LAUNCH_DEPENDENT(gemm_i8_ares_kernel<PACKED>, dim3(grid), dim3(threads_of<PACKED>()), SMEM, s, ta, tb, tc,
                        a_scale, w_scale, out_scale, M, N, K, epi, groups);
    return MI_OK;
}

// The 2-SM kernel for int8 weights and an output of N % 256 == 0 with at least one
// 256 x 256 tile per SM pair; MI_GEMM_2SM=0 in the environment selects the one-CTA
// kernels instead (read per call, for comparisons and tests).
static bool use_pair_kernel(bool packed, int M, int N, int sms) {
    if (packed) return false;
    const char* e = getenv("MI_GEMM_2SM");
    if (e && e[0] == '0') return false;
    return N % BN2 == 0 && (long long)cdiv(M, BM2) * (N / BN2) >= sms / 2;
}

// Shape checks shared by both weight formats, then the kernel choice.
template <bool PACKED>
static int bitlinear(const int8_t* A, int lda, const void* W, const float* a_scale, const float* w_scale,
                     const float* out_scale, void* out, int ldo, int M, int N, int K, int epilogue, void* stream) {
    if (!A || !W || !out) return MI_ERR_INVALID;
    if (M <= 0 || N <= 0 || K <= 0) return MI_ERR_INVALID;
    if (epilogue != MI_EPI_I32 && epilogue != MI_EPI_F32_SCALED) return MI_ERR_INVALID;
    if (epilogue == MI_EPI_F32_SCALED && (!a_scale || !w_scale)) return MI_ERR_INVALID;
    if (K % 16 != 0 || lda < K || lda % 16 != 0 || N % 16 != 0) return MI_ERR_UNSUPPORTED;
    if (PACKED && K % 64 != 0) return MI_ERR_UNSUPPORTED;  // packed rows of K/4 bytes: 16-byte pitch for the TMA
    if (ldo < N || ldo % 4 != 0) return MI_ERR_INVALID;
    if ((((uintptr_t)A) | ((uintptr_t)W)) & 15) return MI_ERR_INVALID;
    if (((uintptr_t)out) & 15) return MI_ERR_INVALID;
    if (K > 132104) return MI_ERR_UNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    const int sms = sm_count();
    const long long tm = cdiv(M, BM);
    auto fills = [&](int bn) { return tm * cdiv(N, bn) >= sms; };
    // the pair kernel (256 x 256 tiles over two SMs) for int8 weights wherever N allows it
    // and its tiles give every SM pair work
    if (use_pair_kernel(PACKED, M, N, sms))
        return launch2(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    // 256-wide tiles run the tensor cores at about twice the rate of 128-wide
    // ones; when N allows them they win even though A is then re-read from L2
    // for every N tile.  Otherwise wide outputs over a short K keep A resident.
    const bool wide256 = N % 256 == 0 && fills(256);
    if (!wide256 && K <= ARES_MAXK * BK && N > 128)
        return launch_ares<PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    if (N <= 128 && N % 16 == 0 && N != 128) {
        // narrow projections (x_proj: N = dt_rank + 2*d_state) in one N tile
        if (N <= 32) return launch<32, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        if (N <= 64) return launch<64, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        if (N <= 80) return launch<80, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        if (N <= 96) return launch<96, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        return launch<128, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    }
    // the widest N tile that still gives every SM a tile (few-row GEMMs, e.g.
    // decoding, get narrower tiles and more CTAs)
    if (wide256 && PACKED && K >= 1536)  // tensor-bound packed shapes: the HEAVY setting
        return launch<256, PACKED, true>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    if (wide256)
        return launch<256, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    // A GEMM of a few row tiles (decoding) is latency-bound: one wave of 64-wide tiles
    // on at least half the SMs beats two waves of 32-wide ones (256 decode streams:
    // in_proj 256 -> 128 tiles, 1.420 -> 1.376 ms per step)
    auto one_wave = [&](int bn) {
        const long long t = tm * cdiv(N, bn);
        return t <= sms && 2 * t >= sms;
    };
    if (!fills(128) && one_wave(64))
        return launch<64, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    if (fills(128))
        return launch<128, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    if (fills(64))
        return launch<64, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    return launch<32, PACKED>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
}

// Dense int8 ternary rows -> the 2-bit format (one thread per 16-weight word).
// A value outside {-1, 0, 1} is stored as 0 and sets MI_DEV_PRECOND.
__global__ void pack_ternary_kernel(const int8_t* __restrict__ W, int ldw, uint32_t* __restrict__ Wp, int N,
                                    int K) {
    const int words = K / 16;
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)N * words) return;
    const int n = (int)(i / words), g = (int)(i % words);
    const int4 v = *reinterpret_cast<const int4*>(W + (size_t)n * ldw + 16 * g);
    const int8_t* b = reinterpret_cast<const int8_t*>(&v);
    uint32_t w = 0;
    bool bad = false;
#pragma unroll
    for (int e = 0; e < 16; e++) {
        const int x = b[e];
        bad |= (x < -1 || x > 1);
        const uint32_t code = (x >= -1 && x <= 1) ? ((uint32_t)x & 3u) : 0u;
        const int q = e >> 2, j = e & 3;  // weight 4q + j of the group
        w |= code << (4 * j + 2 * (q & 1) + 16 * (q >> 1));
    }
    if (bad) raise_dev_error(MI_DEV_PRECOND);
    Wp[i] = w;
}

}  // namespace gemm
}  // namespace mi

extern "C" int mi_pack_ternary(const int8_t* W, int ldw, uint8_t* Wp, int N, int K, void* stream) {
    using namespace mi::gemm;
    if (!W || !Wp || N <= 0 || K <= 0 || ldw < K) return MI_ERR_INVALID;
    if (K % 16 != 0 || ldw % 16 != 0) return MI_ERR_UNSUPPORTED;
    if ((((uintptr_t)W) & 15) || (((uintptr_t)Wp) & 3)) return MI_ERR_INVALID;
    const long long words = (long long)N * (K / 16);
    const int threads = 256;
    pack_ternary_kernel<<<(unsigned)((words + threads - 1) / threads), threads, 0, (cudaStream_t)stream>>>(
        W, ldw, reinterpret_cast<uint32_t*>(Wp), N, K);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

namespace mi {
namespace gemm {

// ---------------------------------------------------------------------------
// BitLinear + BitShift norm + squareplus (BASELINE config 3's epilogue).
//
// The norm of an output row needs statistics of the whole row (8192 columns
// at config 3 = 32 tiles of 256), which no single tile's epilogue sees.  Two
// passes:
//   1. the GEMM (gemm_i8_kernel with row_stats) writes the int32 accumulators
//      and, per tile, adds each row's exact sums S1 = sum acc and
//      S2 = sum acc^2 (int64) into a caller workspace by atomics -- integer
//      sums, so their value does not depend on the tile order;
//   2. norm_sqp_rows_kernel, one warp per row, turns S1, S2 into the mean and
//      the power-of-two scale (double arithmetic on exact integers, each
//      operation rounded once) and streams the row once: dequantise, centre,
//      scale, gamma, step, ste_clamp(-50, 50), squareplus -> fp32.
// The definition (no reference function fuses these stages) is restated in
// oracle/mi_oracle.c:orc_bitlinear_norm_sqp.
// ---------------------------------------------------------------------------

// _find_power_of_2_scale's threshold table (src/mamba_integer_model.py:144-184)
// on a double argument that already includes the 1e-9.
__device__ __forceinline__ float pow2_scale_d(double v) {
    float s = 1.0f;
    if (v >= 4.0) s = 0.5f;
    if (v >= 16.0) s = 0.25f;
    if (v >= 64.0) s = 0.125f;
    if (v >= 256.0) s = 0.0625f;
    if (v >= 1024.0) s = 0.03125f;
    if (v >= 4096.0) s = 0.015625f;
    if (v >= 16384.0) s = 0.0078125f;
    if (v >= 65536.0) s = 0.00390625f;
    if (v < 1.0) s = 1.0f;
    if (v < 0.25) s = 2.0f;
    if (v < 0.0625) s = 4.0f;
    if (v < 0.015625) s = 8.0f;
    return s;
}

__device__ __forceinline__ float norm_elem(int32_t a, float sc, float mean, float s, float g, float st) {
    const float y = __fmul_rn(__int2float_rn(a), sc);
    const float xc = __fsub_rn(y, mean);
    return ste_clamp(__fmul_rn(__fmul_rn(__fmul_rn(xc, s), g), st), -50.0f, 50.0f);
}

__global__ void __launch_bounds__(256)
norm_sqp_rows_kernel(const int32_t* __restrict__ acc, int ldc, const unsigned long long* __restrict__ stats,
                     const float* __restrict__ a_scale, const float* __restrict__ w_scale,
                     const float* __restrict__ gamma, const float* __restrict__ step, float* __restrict__ out,
                     int ldo, int M, int N) {
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const float ws = *w_scale, st = *step;
    for (int m = blockIdx.x * warps + (threadIdx.x >> 5); m < M; m += gridDim.x * warps) {
        const long long s1 = (long long)stats[2 * (size_t)m], s2 = (long long)stats[2 * (size_t)m + 1];
        const float sc = __fmul_rn(ws, a_scale[m]);  // (w_scale * x_scale), as the BitLinear rescale
        const double dsc = (double)sc;
        const float mean = __double2float_rn(__dmul_rn(__ddiv_rn(__ll2double_rn(s1), (double)N), dsc));
        const long long vnum = (long long)N * s2 - s1 * s1;  // >= 0, < 2^62 for N*K <= 2^24
        const double var = __dmul_rn(__ddiv_rn(__ll2double_rn(vnum), __dmul_rn((double)N, (double)N)),
                                     __dmul_rn(dsc, dsc));
        const float s = pow2_scale_d(__dadd_rn(var, (double)1e-9f));
        const int32_t* row = acc + (size_t)m * ldc;
        float* orow = out + (size_t)m * ldo;
        for (int c = 4 * lane; c < N; c += 128) {
            const int4 a = *reinterpret_cast<const int4*>(row + c);
            const float4 g = *reinterpret_cast<const float4*>(gamma + c);
            // ste_clamp results (not f32x2 products) feed the paired squareplus
            const float2 p = squareplus_bounded2(make_float2(norm_elem(a.x, sc, mean, s, g.x, st),
                                                             norm_elem(a.y, sc, mean, s, g.y, st)));
            const float2 q = squareplus_bounded2(make_float2(norm_elem(a.z, sc, mean, s, g.z, st),
                                                             norm_elem(a.w, sc, mean, s, g.w, st)));
            *reinterpret_cast<float4*>(orow + c) = make_float4(p.x, p.y, q.x, q.y);
        }
    }
}

static int bitlinear_norm_sqp(const int8_t* A, int lda, const uint8_t* Wp, const float* a_scale,
                              const float* w_scale, const float* gamma, const float* step, int32_t* acc, int ldc,
                              float* out, int ldo, unsigned long long* stats_ws, int M, int N, int K,
                              cudaStream_t s) {
    if (!A || !Wp || !a_scale || !w_scale || !gamma || !step || !acc || !out || !stats_ws) return MI_ERR_INVALID;
    if (M <= 0 || N <= 0 || K <= 0) return MI_ERR_INVALID;
    if (K % 64 != 0 || lda < K || lda % 16 != 0 || N % 16 != 0) return MI_ERR_UNSUPPORTED;
    if ((long long)N * K > (1LL << 24)) return MI_ERR_UNSUPPORTED;  // keeps N*S2 and S1^2 below 2^62
    if (ldc < N || ldc % 4 != 0 || ldo < N || ldo % 4 != 0) return MI_ERR_INVALID;
    if ((((uintptr_t)A) | ((uintptr_t)Wp) | ((uintptr_t)acc) | ((uintptr_t)out) | ((uintptr_t)gamma)) & 15)
        return MI_ERR_INVALID;
    if (((uintptr_t)stats_ws) & 7) return MI_ERR_INVALID;
    if (cudaMemsetAsync(stats_ws, 0, sizeof(unsigned long long) * 2 * (size_t)M, s) != cudaSuccess) {
        cudaGetLastError();
        return MI_ERR_CUDA;
    }
    const int sms = sm_count();
    const long long tm = cdiv(M, BM);
    auto fills = [&](int bn) { return tm * cdiv(N, bn) >= sms; };
    int rc;
    // the streaming kernel (its epilogue adds the row sums), widest tile that fills the SMs
    if (N <= 32) rc = launch<32, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else if (N <= 64) rc = launch<64, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else if (N <= 96) rc = launch<96, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else if (N % 256 == 0 && fills(256) && K >= 1536)
        rc = launch<256, true, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else if (N % 256 == 0 && fills(256))
        rc = launch<256, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else if (N <= 128 || fills(128))
        rc = launch<128, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else if (fills(64))
        rc = launch<64, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    else
        rc = launch<32, true>(A, lda, Wp, a_scale, w_scale, nullptr, acc, ldc, M, N, K, MI_EPI_I32, s, stats_ws);
    if (rc != MI_OK) return rc;
    int blocks = cdiv(M, 8);
    if (blocks > sms * 16) blocks = sms * 16;
    norm_sqp_rows_kernel<<<blocks, 256, 0, s>>>(acc, ldc, stats_ws, a_scale, w_scale, gamma, step, out, ldo, M, N);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

}  // namespace gemm
}  // namespace mi

extern "C" int mi_bitlinear_packed_norm_sqp(const int8_t* A, int lda, const uint8_t* Wp, const float* a_scale,
                                            const float* w_scale, const float* gamma, const float* step,
                                            int32_t* acc, int ldc, float* out, int ldo, uint64_t* stats_ws, int M,
                                            int N, int K, void* stream) {
    return mi::gemm::bitlinear_norm_sqp(A, lda, Wp, a_scale, w_scale, gamma, step, acc, ldc, out, ldo,
                                        reinterpret_cast<unsigned long long*>(stats_ws), M, N, K,
                                        (cudaStream_t)stream);
}

extern "C" int mi_bitlinear_packed(const int8_t* A, int lda, const uint8_t* Wp, const float* a_scale,
                                   const float* w_scale, const float* out_scale, void* out, int ldo, int M, int N,
                                   int K, int epilogue, void* stream) {
    return mi::gemm::bitlinear<true>(A, lda, Wp, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, stream);
}

extern "C" int mi_bitlinear_i8(const int8_t* A, int lda, const int8_t* W, const float* a_scale, const float* w_scale,
                               const float* out_scale, void* out, int ldo, int M, int N, int K, int epilogue,
                               void* stream) {
    return mi::gemm::bitlinear<false>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, stream);
}
