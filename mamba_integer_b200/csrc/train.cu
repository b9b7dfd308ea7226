// train.cu -- training-side passes of the path: the backward of the convex
// dyadic scan and the straight-through backward of the per-token int8
// activation quantisation.
//
// Both restate the reference's arithmetic operation by operation (fp32, each
// operation rounded once, no contraction), so their results are the bits the
// reference's own CPU code gives; tests/golden/backward.npz holds vectors that
// code produced.
#include "mi_common.cuh"

namespace mi {
namespace train {

// Convex scan backward, one thread per (sequence, channel) walking t from the
// end (the accumulation is a recurrence in t):
//   g[t] = grad_h[t] + decay[t] * g[t+1]          decay = nums / 32768
//   grad_u[t] = (1 - decay[t]) * g[t]
//   grad_nums[t] = (g[t] * (h[t-1] - u[t])) / 32768   (h[-1] = 0)
// (src/mamba_integer_model.py:319-344; the Triton fast backward
// src/triton_kernels/dyadic_scan.py:376-459 computes the same quantities in a
// parallel order).  Threads of a warp take adjacent channels, so every load
// and store of a step is one coalesced row segment; the loads of UNR steps are
// issued before their recurrence, which only depends on g.
constexpr int BWD_THREADS = 128;
constexpr int UNR = 4;

__global__ void __launch_bounds__(BWD_THREADS)
scan_convex_bwd_kernel(const float* __restrict__ grad_h, const float* __restrict__ h, const float* __restrict__ u,
                       const float* __restrict__ nums, float* __restrict__ grad_u, float* __restrict__ grad_nums,
                       int L, int DN) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int b = blockIdx.y;
    if (c >= DN) return;
    const size_t base = (size_t)b * L * DN + c;
    float acc = 0.0f;
    int t = L - 1;
    for (; t >= UNR - 1; t -= UNR) {
        float gh[UNR], nm[UNR], uu[UNR], hp[UNR];
#pragma unroll
        for (int j = 0; j < UNR; j++) {
            const int tt = t - j;
            const size_t o = base + (size_t)tt * DN;
            gh[j] = grad_h[o];
            nm[j] = nums[o];
            uu[j] = u[o];
            hp[j] = tt > 0 ? h[o - DN] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < UNR; j++) {
            const size_t o = base + (size_t)(t - j) * DN;
            const float d = __fdiv_rn(nm[j], 32768.0f);
            acc = __fadd_rn(gh[j], __fmul_rn(d, acc));
            grad_u[o] = __fmul_rn(__fsub_rn(1.0f, d), acc);
            grad_nums[o] = __fdiv_rn(__fmul_rn(acc, __fsub_rn(hp[j], uu[j])), 32768.0f);
        }
    }
    for (; t >= 0; t--) {
        const size_t o = base + (size_t)t * DN;
        const float d = __fdiv_rn(nums[o], 32768.0f);
        acc = __fadd_rn(grad_h[o], __fmul_rn(d, acc));
        grad_u[o] = __fmul_rn(__fsub_rn(1.0f, d), acc);
        const float hp = t > 0 ? h[o - DN] : 0.0f;
        grad_nums[o] = __fdiv_rn(__fmul_rn(acc, __fsub_rn(hp, u[o])), 32768.0f);
    }
}

// Straight-through backward of activation_quant_dynamic's Triton path
// (src/triton_kernels/bitnet_kernels.py:77-95): with the row's saved scale
// amax[t] (its max |x|),
//   grad_x = clamp((grad_xq * 127) / clamp(amax, min=0.01), -100, 100).
// Rows of K values, 4 per thread per 16-byte access when K % 4 == 0.
__global__ void __launch_bounds__(256)
quant_ste_bwd_kernel(const float* __restrict__ gq, const float* __restrict__ amax, float* __restrict__ gx, int T,
                     int K) {
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
        const float s = max_nan(amax[t], 0.01f);  // torch.clamp(min=0.01): NaN stays NaN
        const float* g = gq + (size_t)t * K;
        float* o = gx + (size_t)t * K;
        if ((K & 3) == 0) {
            for (int k = 4 * lane; k < K; k += 128) {
                const float4 v = *reinterpret_cast<const float4*>(g + k);
                float4 r;
                r.x = clamp_t(__fdiv_rn(__fmul_rn(v.x, 127.0f), s), -100.0f, 100.0f);
                r.y = clamp_t(__fdiv_rn(__fmul_rn(v.y, 127.0f), s), -100.0f, 100.0f);
                r.z = clamp_t(__fdiv_rn(__fmul_rn(v.z, 127.0f), s), -100.0f, 100.0f);
                r.w = clamp_t(__fdiv_rn(__fmul_rn(v.w, 127.0f), s), -100.0f, 100.0f);
                *reinterpret_cast<float4*>(o + k) = r;
            }
        } else {
            for (int k = lane; k < K; k += 32) o[k] = clamp_t(__fdiv_rn(__fmul_rn(g[k], 127.0f), s), -100.0f, 100.0f);
        }
    }
}

}  // namespace train
}  // namespace mi

extern "C" int mi_scan_convex_backward(const float* grad_h, const float* h, const float* u, const float* nums,
                                       float* grad_u, float* grad_nums, int batch, int L, int DN, void* stream) {
    if (!grad_h || !h || !u || !nums || !grad_u || !grad_nums) return MI_ERR_INVALID;
    if (batch <= 0 || L <= 0 || DN <= 0) return MI_ERR_INVALID;
    if (batch > 65535) return MI_ERR_UNSUPPORTED;
    dim3 grid(mi::cdiv(DN, mi::train::BWD_THREADS), batch);
    mi::train::scan_convex_bwd_kernel<<<grid, mi::train::BWD_THREADS, 0, (cudaStream_t)stream>>>(
        grad_h, h, u, nums, grad_u, grad_nums, L, DN);
    MI_CHECK_LAUNCH();
    return MI_OK;
}

extern "C" int mi_quant_ste_backward(const float* grad_xq, const float* amax, float* grad_x, int T, int K,
                                     void* stream) {
    if (!grad_xq || !amax || !grad_x) return MI_ERR_INVALID;
    if (T < 0 || K <= 0) return MI_ERR_INVALID;
    if (T == 0) return MI_OK;
    if ((K & 3) == 0 && ((((uintptr_t)grad_xq) | ((uintptr_t)grad_x)) & 15)) return MI_ERR_INVALID;
    int blocks = mi::cdiv(T, 8);
    if (blocks > 148 * 16) blocks = 148 * 16;
    mi::train::quant_ste_bwd_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(grad_xq, amax, grad_x, T, K);
    MI_CHECK_LAUNCH();
    return MI_OK;
}
