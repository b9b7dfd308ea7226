// mi_common.cuh -- shared device helpers for the sm_100a Mamba-Integer kernels.
// Included once by the unity translation unit mi_b200_unity.cu.
//
// Floating-point stages reproduce the reference CPU path operation by
// operation.  Every product and sum below is written with an explicit
// round-to-nearest intrinsic so that no build flag can contract a*b+c into a
// fused multiply-add; the only FMAs are the ones written as __fmaf_rn, at the
// places where the reference itself accumulates with FMA (conv taps, h.C).
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cuda_runtime.h>

#include "../../include/mi_b200.h"

namespace mi {

// per-device error word (bits MI_DEV_*), read by mi_device_error().  The
// library is built as one translation unit (mi_b200_unity.cu), so this is
// the single definition.
__device__ int g_dev_error;

__device__ __forceinline__ void raise_dev_error(int bits) { atomicOr(&g_dev_error, bits); }

// NaN-propagating min / max (PTX min.NaN / max.NaN), as torch.minimum/maximum.
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// torch.clamp(x, lo, hi) on fp32: NaN propagates.  (The sign of a zero result
// can differ from ATen's, which never matters downstream: every clamp here is
// followed by arithmetic that maps +-0 to the same value, or by an int cast.)
__device__ __forceinline__ float clamp_t(float x, float lo, float hi) { return min_nan(max_nan(x, lo), hi); }

// ste_clamp forward value x + (clamp(x) - x)  (src/mamba_integer_model.py:136-141)
__device__ __forceinline__ float ste_clamp(float x, float lo, float hi) {
    float c = clamp_t(x, lo, hi);
    return __fadd_rn(x, __fsub_rn(c, x));
}

// _rsqrt_newton (src/mamba_integer_model.py:80-102): guess table, 3 Newton
// steps r = r * (1.5 - ((0.5*y)*r)*r), each clamped to [1e-6, 1e3].
__device__ __forceinline__ float rsqrt_newton(float y) {
    y = clamp_t(y, 1e-6f, 1e6f);
    float r = (y > 16.0f) ? 0.125f : 0.5f;
    if (y > 64.0f) r = 0.0625f;
    if (y > 256.0f) r = 0.03125f;
    if (y < 4.0f) r = 1.0f;
    if (y < 1.0f) r = 2.0f;
    if (y < 0.25f) r = 4.0f;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        float t = __fmul_rn(0.5f, y);
        t = __fmul_rn(t, r);
        t = __fmul_rn(t, r);
        t = __fsub_rn(1.5f, t);
        r = __fmul_rn(r, t);
        r = clamp_t(r, 1e-6f, 1e3f);
    }
    return r;
}

// _rsqrt_newton for an argument known to be >= 4 or NaN (x*x + 4 always is):
// the three "y < 4 / 1 / 0.25" entries of the guess table can never fire, so
// they are skipped; every other operation is the same as rsqrt_newton.
__device__ __forceinline__ float rsqrt_newton_ge4(float y) {
    y = clamp_t(y, 1e-6f, 1e6f);
    float r = (y > 16.0f) ? 0.125f : 0.5f;
    r = (y > 64.0f) ? 0.0625f : r;
    r = (y > 256.0f) ? 0.03125f : r;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        float t = __fmul_rn(0.5f, y);
        t = __fmul_rn(t, r);
        t = __fmul_rn(t, r);
        t = __fsub_rn(1.5f, t);
        r = __fmul_rn(r, t);
        r = clamp_t(r, 1e-6f, 1e3f);
    }
    return r;
}

// _squareplus_rational (src/mamba_integer_model.py:105-121)
__device__ __forceinline__ float squareplus(float x) {
    float ysq = __fadd_rn(__fmul_rn(x, x), 4.0f);  // >= 4 or NaN
    float ys = clamp_t(ysq, 1e-6f, 1e6f);
    float r = rsqrt_newton_ge4(ys);
    float s = clamp_t(__fmul_rn(ys, r), 0.0f, 1e3f);
    return __fmul_rn(0.5f, __fadd_rn(x, s));
}

// squareplus of an argument known to satisfy |x| <= 999 or to be NaN: then
// x*x + 4 lies in [4, 1e6] or is NaN, and the two clamps to [1e-6, 1e6] in
// front of the Newton iteration are identities, so they are skipped.  Same
// result as squareplus() for every such argument.  The outputs of
// ste_clamp(., -50, 50) and ste_clamp(., -20, 20) qualify: x + (c - x)
// differs from c by at most half an ulp of x, and when that exceeds the bound
// the difference c - x rounds to -x and the result is 0, so the magnitude
// never exceeds 2 * 50.
// The upper clamp of each Newton step (r <= 1e3) is skipped too: y > 0 and
// r > 0 make t = (0.5*y*r)*r >= 0, so 1.5 - t <= 1.5 and each step at most
// multiplies r by fl(1.5); from a guess <= 0.5, r stays below 1.7 after three
// steps.  A NaN or +inf y gives the same r with or without it (NaN, and the
// lower clamp 1e-6, respectively).
__device__ __forceinline__ float squareplus_bounded(float x) {
    const float y = __fadd_rn(__fmul_rn(x, x), 4.0f);
    float r = (y > 16.0f) ? 0.125f : 0.5f;
    r = (y > 64.0f) ? 0.0625f : r;
    r = (y > 256.0f) ? 0.03125f : r;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        float t = __fmul_rn(0.5f, y);
        t = __fmul_rn(t, r);
        t = __fmul_rn(t, r);
        t = __fsub_rn(1.5f, t);
        r = __fmul_rn(r, t);
        r = max_nan(r, 1e-6f);  // the upper clamp never binds here (see above)
    }
    const float s = clamp_t(__fmul_rn(y, r), 0.0f, 1e3f);
    return __fmul_rn(0.5f, __fadd_rn(x, s));
}

// Two independent elements at once with f32x2 operations (each component
// rounds exactly as the scalar operation).  An f32x2 add or FMA whose operand
// is an f32x2 product is contracted by the compiler (dropping the product's
// rounding), so every addition that follows a product stays scalar; additions
// of clamp results (min/max outputs) are safe.
//
// ste_clamp of a pair that is NOT an f32x2 product (its two adds would be
// fused with the product); clamp results and FMA sums are fine.
__device__ __forceinline__ float2 ste_clamp2(float2 x, float lo, float hi) {
    const float2 c = make_float2(clamp_t(x.x, lo, hi), clamp_t(x.y, lo, hi));
    const float2 d = __fadd2_rn(c, make_float2(-x.x, -x.y));  // clamp(x) - x
    return __fadd2_rn(x, d);
}

// squareplus_bounded of a pair
__device__ __forceinline__ float2 squareplus_bounded2(float2 x) {
    const float2 xx = __fmul2_rn(x, x);
    const float2 y = make_float2(__fadd_rn(xx.x, 4.0f), __fadd_rn(xx.y, 4.0f));
    float2 r;
    r.x = (y.x > 16.0f) ? 0.125f : 0.5f;
    r.x = (y.x > 64.0f) ? 0.0625f : r.x;
    r.x = (y.x > 256.0f) ? 0.03125f : r.x;
    r.y = (y.y > 16.0f) ? 0.125f : 0.5f;
    r.y = (y.y > 64.0f) ? 0.0625f : r.y;
    r.y = (y.y > 256.0f) ? 0.03125f : r.y;
    const float2 half = make_float2(0.5f, 0.5f);
#pragma unroll
    for (int i = 0; i < 3; i++) {
        float2 t = __fmul2_rn(half, y);
        t = __fmul2_rn(t, r);
        t = __fmul2_rn(t, r);
        t = make_float2(__fsub_rn(1.5f, t.x), __fsub_rn(1.5f, t.y));
        r = __fmul2_rn(r, t);
        r = make_float2(max_nan(r.x, 1e-6f), max_nan(r.y, 1e-6f));  // as in squareplus_bounded
    }
    const float2 p = __fmul2_rn(y, r);
    const float2 sq = make_float2(clamp_t(p.x, 0.0f, 1e3f), clamp_t(p.y, 0.0f, 1e3f));
    return __fmul2_rn(half, __fadd2_rn(x, sq));
}

// y * _sigmoid_algebraic(z) = y * (0.5 + (0.5*z) / (1 + |z|))  (:124-132, :444)
__device__ __forceinline__ float sigmoid_gate(float y, float z) {
    float num = __fmul_rn(0.5f, z);
    float den = __fadd_rn(1.0f, fabsf(z));
    float s = __fadd_rn(0.5f, __fdiv_rn(num, den));
    return __fmul_rn(y, s);
}

// _find_power_of_2_scale (src/mamba_integer_model.py:144-184)
__device__ __forceinline__ float pow2_scale(float var) {
    float v = __fadd_rn(var, 1e-9f);
    float s = 1.0f;
    if (v >= 4.0f) s = 0.5f;
    if (v >= 16.0f) s = 0.25f;
    if (v >= 64.0f) s = 0.125f;
    if (v >= 256.0f) s = 0.0625f;
    if (v >= 1024.0f) s = 0.03125f;
    if (v >= 4096.0f) s = 0.015625f;
    if (v >= 16384.0f) s = 0.0078125f;
    if (v >= 65536.0f) s = 0.00390625f;
    if (v < 1.0f) s = 1.0f;
    if (v < 0.25f) s = 2.0f;
    if (v < 0.0625f) s = 4.0f;
    if (v < 0.015625f) s = 8.0f;
    return s;
}

// activation_quant_dynamic's scale (src/rational_bitnet.py:102-111) from a
// row's max |x|: s = max(amax, 1e-8) (NaN propagates), xscale = s / 127, and
// the multiplier 127 / s computed as Tensor.__rdiv__ does: reciprocal(s) * 127.
__device__ __forceinline__ float quant_inv_scale(float amax, float& xscale) {
    const float sc = clamp_t(amax, 1e-8f, __int_as_float(0x7f800000));
    xscale = __fdiv_rn(sc, 127.0f);
    return __fmul_rn(__frcp_rn(sc), 127.0f);
}

// int8 value of clamp(ste_round(v), -127, 127), ste_round(v) = v + (rne(v) - v)
// (src/rational_bitnet.py:54-60, :109)
__device__ __forceinline__ int quant_i8(float v) {
    float r = rintf(v);
    float q = __fadd_rn(v, __fsub_rn(r, v));
    q = clamp_t(q, -127.0f, 127.0f);
    return (int)q;
}

// ceil(a / b) for positive ints
__host__ __device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// Programmatic dependent launch.  A kernel started by launch_dependent() may
// begin while the kernel before it in the stream is still finishing (its
// launch and prologue overlap that kernel's tail).  Such a kernel calls
// grid_dependency_sync() before its first access to global memory that an
// earlier kernel writes, or reads and this kernel then overwrites: it returns
// once every earlier kernel has completed and its writes are visible.  The
// kernel then lets its own successor start launching; as that successor
// waits in the same way, at most two kernels of the stream overlap.  In a
// kernel launched without the attribute both instructions have nothing to
// wait for.
__device__ __forceinline__ void grid_dependency_sync() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// MI_PDL=0 in the environment launches every kernel fully serialised (read
// once per process, at the first launch: a getenv per launch costs host time
// in the eager, launch-bound paths).
static inline bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("MI_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                           cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace mi

#define MI_CHECK_LAUNCH()                                   \
    do {                                                    \
        cudaError_t e_ = cudaGetLastError();                \
        if (e_ != cudaSuccess) return MI_ERR_CUDA;          \
    } while (0)

// mi::launch_dependent(kernel, grid, block, smem, stream, args...) or return MI_ERR_CUDA
#define MI_LAUNCH_DEPENDENT(...)                                   \
    do {                                                           \
        if (mi::launch_dependent(__VA_ARGS__) != cudaSuccess) {    \
            cudaGetLastError();                                    \
            return MI_ERR_CUDA;                                    \
        }                                                          \
    } while (0)
