// gemm_i8.cu -- ternary BitLinear contraction on the 5th-generation tensor
// cores: C[m,n] = sum_k A[m,k] * W[n,k] with A the int8 activations and W the
// ternary weights stored as int8, tcgen05.mma kind::i8 with int32
// accumulators in tensor memory.
//
// Per CTA one BM x BN output tile (BM = 128 rows of tokens):
//   warp 0 / lane 0  TMA producer: 2-D tiled loads (128-byte swizzle) of the
//                    A and W K-slices into a STAGES-deep shared-memory ring;
//   warp 1 / lane 0  MMA issuer: 4 x tcgen05.mma (K = 32 bytes each) per
//                    128-byte K-slice, tcgen05.commit frees the slot;
//   all 4 warps      epilogue: tcgen05.ld 32x32b (one accumulator row per
//                    thread), dequantise acc * (w_scale * a_scale[m])
//                    [* out_scale] exactly as BitLinear.forward does
//                    (src/rational_bitnet.py:204-208), store.
// Every mbarrier wait is bounded (about 2 s of clock); on expiry the CTA sets
// MI_DEV_TIMEOUT, stops issuing, frees its tensor memory and exits.
//
// The accumulation is exact: |sum| <= 127*K < 2^31, and int -> fp32 is exact
// below 2^24 (K <= 132104), the range every BitLinear of the model is in.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "mi_common.cuh"

namespace mi {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes (= int8 elements) of K per stage: one 128-byte swizzle row
constexpr int THREADS = 128;
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s at 2 GHz

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN >= 256 ? 4 : (BN >= 128 ? 3 : 4);
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
    static_assert(STAGE_BYTES % 1024 == 0, "stage must keep 1024-byte alignment for the 128B swizzle");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
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

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const float* __restrict__ a_scale, const float* __restrict__ w_scale,
               const float* __restrict__ out_scale, void* __restrict__ out, int ldo, int M, int N, int K, int epi) {
    using C = Cfg<BN>;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-aligned tiles
    unsigned char* gbase = smem_raw + (base - raw);
    const uint32_t bars = base + C::STAGES * C::STAGE_BYTES;
    // barrier block: full[S], empty[S], accum, then tmem slot and abort flag
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
    const uint32_t accum_bar = bars + 8u * (2 * C::STAGES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::STAGES * C::STAGE_BYTES + 8 * (2 * C::STAGES + 1));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * BM;
    const int num_k = cdiv(K, BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(accum_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        for (int i = 0; i < num_k; i++) {
            const int s = i % C::STAGES;
            if (i >= C::STAGES) {
                if (!mbar_wait(empty_bar(s), ((i / C::STAGES) - 1) & 1, abort_flag)) break;
            }
            const uint32_t sa = base + s * C::STAGE_BYTES;
            mbar_expect_tx(full_bar(s), C::STAGE_BYTES);
            tma_load_2d(sa, &tmA, full_bar(s), i * BK, m0);
            tma_load_2d(sa + C::A_BYTES, &tmB, full_bar(s), i * BK, n0);
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t idesc = idesc_i8<BN>();
        bool ok = true;
        for (int i = 0; i < num_k; i++) {
            const int s = i % C::STAGES;
            if (!mbar_wait(full_bar(s), (i / C::STAGES) & 1, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sa = base + s * C::STAGE_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 32; kk++) {
                const uint64_t ad = sdesc_sw128(sa + kk * 32);
                const uint64_t bd = sdesc_sw128(sa + C::A_BYTES + kk * 32);
                mma_i8(tmem, ad, bd, idesc, (i | kk) != 0);
            }
            mma_commit(empty_bar(s));
        }
        if (ok) mma_commit(accum_bar);
    }
    __syncwarp();

    // ---------------- epilogue ----------------
    const bool have = __all_sync(0xffffffffu, mbar_wait(accum_bar, 0, abort_flag));
    tc_fence_after();
    if (have) {
        const int row = m0 + warp * 32 + lane;
        const bool row_ok = row < M;
        float sc = 0.0f, os = 1.0f;
        if (epi == MI_EPI_F32_SCALED && row_ok) {
            sc = __fmul_rn(*w_scale, a_scale[row]);  // (w_scale * x_scale)
            if (out_scale) os = *out_scale;
        }
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
            const int col = n0 + c0;
            if (!row_ok || col >= N) continue;
            if (epi == MI_EPI_I32) {
                int32_t* o = reinterpret_cast<int32_t*>(out) + (size_t)row * ldo + col;
                if (col + 16 <= N) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<int4*>(o + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                } else {
                    for (int j = 0; j < 16 && col + j < N; j++) o[j] = (int32_t)r[j];
                }
            } else {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    v[j] = __fmul_rn((float)(int32_t)r[j], sc);
                    if (out_scale) v[j] = __fmul_rn(v[j], os);
                }
                float* o = reinterpret_cast<float*>(out) + (size_t)row * ldo + col;
                if (col + 16 <= N) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
                    for (int j = 0; j < 16 && col + j < N; j++) o[j] = v[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"((uint32_t)C::TMEM_COLS)
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

// 2-D int8 tensor [rows, cols] with row pitch ld bytes; box = 128 bytes x box_rows.
static int make_tmap(CUtensorMap* tm, const void* ptr, int rows, int cols, int ld, int box_rows) {
    auto enc = get_encode();
    if (!enc) return MI_ERR_CUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MI_OK : MI_ERR_CUDA;
}

template <int BN>
static int launch(const int8_t* A, int lda, const int8_t* W, const float* a_scale, const float* w_scale,
                  const float* out_scale, void* out, int ldo, int M, int N, int K, int epi, cudaStream_t s) {
    CUtensorMap ta, tb;
    int rc = make_tmap(&ta, A, M, K, lda, BM);
    if (rc) return rc;
    rc = make_tmap(&tb, W, N, K, K, BN);
    if (rc) return rc;
    using C = Cfg<BN>;
    if (cudaFuncSetAttribute(gemm_i8_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
        return MI_ERR_CUDA;
    dim3 grid(cdiv(N, BN), cdiv(M, BM));
    gemm_i8_kernel<BN><<<grid, THREADS, C::SMEM, s>>>(ta, tb, a_scale, w_scale, out_scale, out, ldo, M, N, K, epi);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

}  // namespace gemm
}  // namespace mi

extern "C" int mi_bitlinear_i8(const int8_t* A, int lda, const int8_t* W, const float* a_scale, const float* w_scale,
                               const float* out_scale, void* out, int ldo, int M, int N, int K, int epilogue,
                               void* stream) {
    using namespace mi::gemm;
    if (!A || !W || !out) return MI_ERR_INVALID;
    if (M <= 0 || N <= 0 || K <= 0) return MI_ERR_INVALID;
    if (epilogue != MI_EPI_I32 && epilogue != MI_EPI_F32_SCALED) return MI_ERR_INVALID;
    if (epilogue == MI_EPI_F32_SCALED && (!a_scale || !w_scale)) return MI_ERR_INVALID;
    if (K % 16 != 0 || lda < K || lda % 16 != 0 || N % 16 != 0) return MI_ERR_UNSUPPORTED;
    if (ldo < N || ldo % 4 != 0) return MI_ERR_INVALID;
    if ((((uintptr_t)A) | ((uintptr_t)W)) & 15) return MI_ERR_INVALID;
    if (((uintptr_t)out) & 15) return MI_ERR_INVALID;
    if (K > 132104) return MI_ERR_UNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    if (N <= 128 && N % 16 == 0 && N != 128) {
        // narrow projections (x_proj: N = dt_rank + 2*d_state) in one N tile
        if (N <= 32) return launch<32>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        if (N <= 64) return launch<64>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        if (N <= 80) return launch<80>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        if (N <= 96) return launch<96>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
        return launch<128>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
    }
    return launch<128>(A, lda, W, a_scale, w_scale, out_scale, out, ldo, M, N, K, epilogue, s);
}
