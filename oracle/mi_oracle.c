/*
 * mi_oracle.c -- CPU restatement of the Mamba-Integer inference hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the CUDA
 * kernels in mamba_integer_b200/csrc and the "port" CPU baseline timed by
 * bench.py.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may
 * load it.  The product path never calls into it.
 *
 * Every function restates one stage of the reference CPU path operation by
 * operation, in the same floating-point order, so that its results are
 * bit-identical to the reference on the same inputs.  The order facts it
 * encodes (ATen cascade sum, conv tap order, h.C accumulation order) were
 * measured against torch 2.11 CPU and are pinned by the golden fixtures in
 * tests/golden/.
 *
 * Compile with -ffp-contract=off: a contracted a*b+c would change results.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_ERR_INVALID (-1)
#define ORC_ERR_OVERFLOW (-4)

#ifdef _OPENMP
#define ORC_THREADS(nt) num_threads((nt) > 0 ? (nt) : omp_get_max_threads())
#else
#define ORC_THREADS(nt)
#endif

/* torch.clamp(x, lo, hi) on fp32 with NaN propagation. */
static inline float clamp_t(float x, float lo, float hi) {
    if (x != x) return x;
    if (x < lo) return lo;
    if (x > hi) return hi;
    return x;
}

/* ste_clamp forward value: x + (clamp(x) - x), literal fp32 arithmetic.
 * Reference: src/mamba_integer_model.py:136-141. */
static inline float ste_clamp(float x, float lo, float hi) {
    float c = clamp_t(x, lo, hi);
    return x + (c - x);
}

/* _rsqrt_newton: guess table, 3 Newton steps, clamps.
 * Reference: src/mamba_integer_model.py:80-102. */
static inline float rsqrt_newton(float y) {
    y = clamp_t(y, 1e-6f, 1e6f);
    float r = (y > 16.0f) ? 0.125f : 0.5f;
    if (y > 64.0f) r = 0.0625f;
    if (y > 256.0f) r = 0.03125f;
    if (y < 4.0f) r = 1.0f;
    if (y < 1.0f) r = 2.0f;
    if (y < 0.25f) r = 4.0f;
    for (int i = 0; i < 3; i++) {
        float t = 0.5f * y;   /* 0.5 * y * r * r evaluates left to right */
        t = t * r;
        t = t * r;
        t = 1.5f - t;
        r = r * t;
        r = clamp_t(r, 1e-6f, 1e3f);
    }
    return r;
}

/* _sqrt_rational: src/mamba_integer_model.py:105-111. */
static inline float sqrt_rational(float y) {
    float ys = clamp_t(y, 1e-6f, 1e6f);
    float r = rsqrt_newton(ys);
    return clamp_t(ys * r, 0.0f, 1e3f);
}

/* _squareplus_rational: 0.5 * (x + sqrt(x*x + 4)).
 * Reference: src/mamba_integer_model.py:114-121. */
static inline float squareplus(float x) {
    float ysq = x * x;
    ysq = ysq + 4.0f;
    float s = sqrt_rational(ysq);
    return 0.5f * (x + s);
}

/* y * _sigmoid_algebraic(z): src/mamba_integer_model.py:124-132, 441-444. */
static inline float sigmoid_gate(float y, float z) {
    float a = fabsf(z);
    float num = 0.5f * z;
    float den = 1.0f + a;
    float s = 0.5f + num / den;
    return y * s;
}

/* _find_power_of_2_scale on one variance value.
 * Reference: src/mamba_integer_model.py:144-184. */
static inline float pow2_scale(float var) {
    float v = var + 1e-9f;
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

static int64_t ceil_log2_i64(int64_t x) {
    if (x <= 2) return 1;
    uint64_t v = (uint64_t)x - 1;
    int64_t last = 0;
    while (v) { last++; v >>= 1; }
    return last;  /* index of the highest set bit of x-1, plus one */
}

/*
 * Row sum in the exact order ATen's CPU cascade_sum uses for a contiguous
 * fp32 row (torch 2.11, 8-lane vectors): 4 interleaved vector accumulators
 * (ILP 4) fed through a 4-level cascade of 2^level_power rows, the vector
 * remainder added into accumulator 0, the 4 accumulators combined in order,
 * then scalar tail elements followed by the 8 vector lanes summed
 * sequentially.  torch.sum / torch.mean(dim=-1) reduce a row this way; mean
 * then divides by the element count.
 */
float orc_aten_sum(const float* x, int64_t D) {
    enum { W = 8, ILP = 4, LEVELS = 4 };
    if (D < W) {
        /* scalar path: ILP-4 scalar accumulators over D/4 rows */
        int64_t size_ilp = D / ILP;
        float acc[ILP] = {0, 0, 0, 0};
        for (int64_t i = 0; i < size_ilp; i++)
            for (int k = 0; k < ILP; k++) acc[k] = acc[k] + x[i * ILP + k];
        for (int64_t i = size_ilp * ILP; i < D; i++) acc[0] = acc[0] + x[i];
        for (int k = 1; k < ILP; k++) acc[0] = acc[0] + acc[k];
        return 0.0f + acc[0];
    }
    int64_t vec_size = D / W;
    int64_t size_ilp = vec_size / ILP;
    int64_t level_power = ceil_log2_i64(size_ilp) / LEVELS;
    if (level_power < 4) level_power = 4;
    int64_t level_step = (int64_t)1 << level_power;
    int64_t level_mask = level_step - 1;
    float acc[LEVELS][ILP][W];
    memset(acc, 0, sizeof(acc));
    int64_t i = 0;
    for (; i + level_step <= size_ilp;) {
        for (int64_t j = 0; j < level_step; ++j, ++i)
            for (int k = 0; k < ILP; k++)
                for (int l = 0; l < W; l++)
                    acc[0][k][l] = acc[0][k][l] + x[(i * ILP + k) * W + l];
        for (int j = 1; j < LEVELS; j++) {
            for (int k = 0; k < ILP; k++)
                for (int l = 0; l < W; l++) {
                    acc[j][k][l] = acc[j][k][l] + acc[j - 1][k][l];
                    acc[j - 1][k][l] = 0.0f;
                }
            int64_t mask = level_mask << (j * level_power);
            if ((i & mask) != 0) break;
        }
    }
    for (; i < size_ilp; ++i)
        for (int k = 0; k < ILP; k++)
            for (int l = 0; l < W; l++)
                acc[0][k][l] = acc[0][k][l] + x[(i * ILP + k) * W + l];
    for (int j = 1; j < LEVELS; j++)
        for (int k = 0; k < ILP; k++)
            for (int l = 0; l < W; l++) acc[0][k][l] = acc[0][k][l] + acc[j][k][l];
    for (int64_t v = size_ilp * ILP; v < vec_size; v++)
        for (int l = 0; l < W; l++) acc[0][0][l] = acc[0][0][l] + x[v * W + l];
    for (int k = 1; k < ILP; k++)
        for (int l = 0; l < W; l++) acc[0][0][l] = acc[0][0][l] + acc[0][k][l];
    float fin = 0.0f;
    for (int64_t t = vec_size * W; t < D; t++) fin = fin + x[t];
    for (int l = 0; l < W; l++) fin = fin + acc[0][0][l];
    return fin;
}

/*
 * BitShiftNorm forward on T rows of D (CPU path):
 *   BitShiftNorm.forward centres once (src/mamba_integer_model.py:462-464),
 *   BitShiftNormFunction.forward centres again and takes var = mean(xc^2)
 *   (:199-205), picks the power-of-2 scale (:218, :144-184) and returns
 *   ((xc * s) * gamma) * step_size (:222).
 * inv_rms (optional) receives s per row.
 */
void orc_bitshift_norm(const float* x, int64_t T, int64_t D, const float* gamma, float step,
                       float* y, float* inv_rms, int nthreads) {
    const float Df = (float)D;
#pragma omp parallel for schedule(static) ORC_THREADS(nthreads)
    for (int64_t t = 0; t < T; t++) {
        const float* xr = x + t * D;
        float* yr = y + t * D;
        float* buf = (float*)malloc(sizeof(float) * (size_t)D);
        float m1 = orc_aten_sum(xr, D) / Df;
        for (int64_t i = 0; i < D; i++) buf[i] = xr[i] - m1;
        float m2 = orc_aten_sum(buf, D) / Df;
        for (int64_t i = 0; i < D; i++) buf[i] = buf[i] - m2;   /* x_centered */
        for (int64_t i = 0; i < D; i++) yr[i] = buf[i] * buf[i]; /* pow(2) */
        float var = orc_aten_sum(yr, D) / Df;
        float s = pow2_scale(var);
        for (int64_t i = 0; i < D; i++) {
            float v = buf[i] * s;
            v = v * gamma[i];
            yr[i] = v * step;
        }
        if (inv_rms) inv_rms[t] = s;
        free(buf);
    }
}

/*
 * activation_quant_dynamic, 8 bits (CPU path, src/rational_bitnet.py:102-111):
 *   s = clamp(amax|x|, min=1e-8); inv = 127 / s, which torch evaluates as
 *   reciprocal(s) * 127 (Tensor.__rdiv__);
 *   xq = clamp(ste_round(x * inv), -127, 127); returns (xq, s / 127).
 * ste_round(v) = v + (round(v) - v) with round half to even (:54-60).
 */
void orc_quant_rows(const float* x, int64_t ldx, int64_t T, int64_t K, int8_t* xq, int64_t ldq,
                    float* xscale, int nthreads) {
#pragma omp parallel for schedule(static) ORC_THREADS(nthreads)
    for (int64_t t = 0; t < T; t++) {
        const float* xr = x + t * ldx;
        float amax = 0.0f;
        int nan = 0;
        for (int64_t k = 0; k < K; k++) {
            float a = fabsf(xr[k]);
            if (a != a) nan = 1;
            if (a > amax) amax = a;
        }
        if (nan) amax = NAN;
        float s = clamp_t(amax, 1e-8f, INFINITY);
        /* `Q_max / scale` is Tensor.__rdiv__: reciprocal(scale) * 127 */
        float inv = (1.0f / s) * 127.0f;
        for (int64_t k = 0; k < K; k++) {
            float v = xr[k] * inv;
            float r = rintf(v);
            float q = v + (r - v);
            q = clamp_t(q, -127.0f, 127.0f);
            xq[t * ldq + k] = (int8_t)q;
        }
        xscale[t] = s / 127.0f;
    }
}

/* weight_quant_ternary given its scale: clamp(ste_round(w / scale), -1, 1).
 * Reference: src/rational_bitnet.py:63-85. */
void orc_ternarize(const float* w, int64_t numel, float scale, int8_t* wq) {
    for (int64_t i = 0; i < numel; i++) {
        float v = w[i] / scale;
        float r = rintf(v);
        float q = clamp_t(v + (r - v), -1.0f, 1.0f);
        wq[i] = (int8_t)q;
    }
}

/*
 * BitLinear matmul + rescale (src/rational_bitnet.py:204-208):
 *   y = F.linear(xq, wq) is an exact integer sum (|y| <= 127*K < 2^24);
 *   out = y * (w_scale * x_scale[t]).
 * acc (optional) receives the int32 accumulators.
 */
void orc_bitlinear(const int8_t* xq, int64_t ldq, const float* xscale, int64_t T, int64_t K,
                   const int8_t* wq, float w_scale, int64_t N, float* out, int64_t ldo,
                   int32_t* acc, int nthreads) {
#pragma omp parallel for schedule(static) ORC_THREADS(nthreads)
    for (int64_t t = 0; t < T; t++) {
        const int8_t* a = xq + t * ldq;
        float sc = w_scale * xscale[t];
        for (int64_t n = 0; n < N; n++) {
            const int8_t* b = wq + n * K;
            int32_t s = 0;
            for (int64_t k = 0; k < K; k++) s += (int32_t)a[k] * (int32_t)b[k];
            if (acc) acc[t * N + n] = s;
            if (out) out[t * ldo + n] = (float)s * sc;
        }
    }
}

/* _find_power_of_2_scale's threshold table (src/mamba_integer_model.py:144-184)
 * on a double argument that already includes the 1e-9. */
static inline float pow2_scale_d(double v) {
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

/*
 * BitLinear epilogue of BASELINE config 3: BitShift norm + squareplus of each
 * output row, statistics taken exactly from the int32 accumulators.  The
 * reference has no fused GEMM + norm; this chains its stages on the BitLinear
 * output y = acc * (w_scale * a_scale[m]) (src/rational_bitnet.py:204-208):
 * BitShiftNorm (src/mamba_integer_model.py:199-222: centre, variance, the
 * power-of-two scale of _find_power_of_2_scale :144-184, ((x_c*s)*gamma)*step),
 * then ste_clamp(-50, 50) and _squareplus_rational (:410-411, :114-121).
 *
 * The reference's fp32 mean and variance depend on its summation order, which
 * a tiled GPU reduction cannot follow, so this build defines them from the
 * exact integer sums S1 = sum acc and S2 = sum acc^2 (int64; N*K <= 2^24 keeps
 * N*S2 and S1^2 below 2^62), with sc = fl(w_scale * a_scale[m]):
 *   mean = (float)((S1 / (double)N) * (double)sc)
 *   var  = ((double)(N*S2 - S1*S1) / ((double)N * N)) * ((double)sc * sc)
 *   s    = pow2 table on var + 1e-9 (double; each double operation rounded once)
 * and one centring (the second centring of BitShiftNormFunction subtracts the
 * mean of an exactly centred row, i.e. zero).  Per element, in fp32:
 *   y = (float)acc * sc;  x_c = y - mean;  o = ((x_c * s) * gamma[n]) * step;
 *   out = squareplus(ste_clamp(o, -50, 50)).
 * stats_out (optional, [M, 2] int64) receives S1, S2.
 */
void orc_bitlinear_norm_sqp(const int32_t* acc, const float* a_scale, float w_scale, const float* gamma, float step,
                            float* out, int64_t* stats_out, int64_t M, int64_t N, int nthreads) {
#pragma omp parallel for schedule(static) ORC_THREADS(nthreads)
    for (int64_t m = 0; m < M; m++) {
        const int32_t* r = acc + m * N;
        int64_t s1 = 0, s2 = 0;
        for (int64_t n = 0; n < N; n++) {
            s1 += r[n];
            s2 += (int64_t)r[n] * r[n];
        }
        if (stats_out) {
            stats_out[2 * m] = s1;
            stats_out[2 * m + 1] = s2;
        }
        const float sc = w_scale * a_scale[m];
        const double dsc = (double)sc;
        const float mean = (float)(((double)s1 / (double)N) * dsc);
        const int64_t vnum = N * s2 - s1 * s1;
        const double var = ((double)vnum / ((double)N * (double)N)) * (dsc * dsc);
        const float s = pow2_scale_d(var + (double)1e-9f);
        for (int64_t n = 0; n < N; n++) {
            const float y = (float)r[n] * sc;
            const float xc = y - mean;
            float o = xc * s;
            o = o * gamma[n];
            o = o * step;
            out[m * N + n] = squareplus(ste_clamp(o, -50.0f, 50.0f));
        }
    }
}

/* Plain int32 GEMM C[m,n] = sum_k A[m,k] W[n,k] (the bare BitLinear contraction). */
void orc_gemm_i8_i32(const int8_t* A, const int8_t* W, int32_t* C, int64_t M, int64_t N, int64_t K,
                     int nthreads) {
#pragma omp parallel for schedule(static) ORC_THREADS(nthreads)
    for (int64_t m = 0; m < M; m++) {
        const int8_t* a = A + m * K;
        for (int64_t n = 0; n < N; n++) {
            const int8_t* b = W + n * K;
            int32_t s = 0;
            for (int64_t k = 0; k < K; k++) s += (int32_t)a[k] * (int32_t)b[k];
            C[m * N + n] = s;
        }
    }
}

/*
 * 2-bit packed storage of ternary weights (this build's own format; the
 * reference keeps the result of weight_quant_ternary, src/rational_bitnet.py:
 * 63-85, as fp32 and exports it as int8, scripts/export_int8.py:77-81).
 * Row n of Wp holds K/4 bytes; the little-endian 32-bit word g of the row
 * holds weights 16g .. 16g+15, weight 16g + 4q + j in bits [p, p+2) with
 * p = 4j + 2(q & 1) + 16(q >> 1), as a 2-bit two's complement value
 * (00 = 0, 01 = +1, 11 = -1).
 * Returns the number of values outside {-1, 0, 1} (stored as 0).
 */
int64_t orc_pack_ternary(const int8_t* W, int64_t N, int64_t K, uint8_t* Wp) {
    int64_t bad = 0;
    for (int64_t n = 0; n < N; n++) {
        for (int64_t g = 0; g < K / 16; g++) {
            uint32_t w = 0;
            for (int e = 0; e < 16; e++) {
                const int x = W[n * K + 16 * g + e];
                uint32_t code = 0;
                if (x == 1) code = 1;
                else if (x == -1) code = 3;
                else if (x != 0) bad++;
                const int q = e >> 2, j = e & 3;
                w |= code << (4 * j + 2 * (q & 1) + 16 * (q >> 1));
            }
            for (int b = 0; b < 4; b++) Wp[n * (K / 4) + 4 * g + b] = (uint8_t)(w >> (8 * b));
        }
    }
    return bad;
}

/* Inverse of orc_pack_ternary: W [N, K] int8 from Wp [N, K/4]. */
void orc_unpack_ternary(const uint8_t* Wp, int64_t N, int64_t K, int8_t* W) {
    for (int64_t n = 0; n < N; n++) {
        for (int64_t k = 0; k < K; k++) {
            const int64_t g = k / 16, e = k % 16;
            const int q = (int)(e >> 2), j = (int)(e & 3);
            const int p = 4 * j + 2 * (q & 1) + 16 * (q >> 1);
            const uint8_t byte = Wp[n * (K / 4) + 4 * g + p / 8];
            const int code = (byte >> (p % 8)) & 3;
            W[n * K + k] = (int8_t)(code == 3 ? -1 : code == 2 ? -2 : code);
        }
    }
}

/*
 * Causal depthwise conv (nn.Conv1d(D, D, 4, groups=D, padding=3), first L
 * outputs; src/mamba_integer_model.py:378, 404) followed by ste_clamp(-50, 50)
 * and _squareplus_rational (:410-411).  The conv accumulates bias first, then
 * one fused multiply-add per tap k = 0..3 over inputs t-3+k.
 * x: [Bsz, L, D] with row stride ldx; conv_out / act_out: [Bsz, L, D] dense
 * (either may be NULL).
 */
void orc_conv_sqp(const float* x, int64_t ldx, int64_t Bsz, int64_t L, int64_t D,
                  const float* w, const float* bias, float* conv_out, float* act_out, int nthreads) {
#pragma omp parallel for collapse(2) schedule(static) ORC_THREADS(nthreads)
    for (int64_t b = 0; b < Bsz; b++)
        for (int64_t t = 0; t < L; t++) {
            for (int64_t d = 0; d < D; d++) {
                float acc = bias[d];
                for (int k = 0; k < 4; k++) {
                    int64_t ti = t - 3 + k;
                    float xv = (ti >= 0) ? x[(b * L + ti) * ldx + d] : 0.0f;
                    acc = fmaf(w[d * 4 + k], xv, acc);
                }
                int64_t o = (b * L + t) * D + d;
                if (conv_out) conv_out[o] = acc;
                if (act_out) act_out[o] = squareplus(ste_clamp(acc, -50.0f, 50.0f));
            }
        }
}

/* Element-wise helpers exposed for stage tests. */
void orc_squareplus_clamp(const float* x, float* y, int64_t n, float lo, float hi) {
    for (int64_t i = 0; i < n; i++) y[i] = squareplus(ste_clamp(x[i], lo, hi));
}
void orc_ste_clamp(const float* x, float* y, int64_t n, float lo, float hi) {
    for (int64_t i = 0; i < n; i++) y[i] = ste_clamp(x[i], lo, hi);
}
void orc_sigmoid_gate(const float* y, const float* z, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = sigmoid_gate(y[i], z[i]);
}

/*
 * DyadicScanFunction forward, CPU branch (src/mamba_integer_model.py:301-315):
 *   decay = nums / 2^15;  h = h * decay + (1 - decay) * u  (4 roundings).
 * u, nums, h: [Bsz, L, DN].
 */
void orc_scan_convex(const float* u, const float* nums, float* h, int64_t Bsz, int64_t L, int64_t DN,
                     int nthreads) {
#pragma omp parallel for collapse(2) schedule(static) ORC_THREADS(nthreads)
    for (int64_t b = 0; b < Bsz; b++)
        for (int64_t c = 0; c < DN; c++) {
            float hv = 0.0f;
            for (int64_t t = 0; t < L; t++) {
                int64_t o = (b * L + t) * DN + c;
                float d = nums[o] / 32768.0f;
                float a = hv * d;
                float om = 1.0f - d;
                float bb = om * u[o];
                hv = a + bb;
                h[o] = hv;
            }
        }
}

/*
 * Backward of the convex dyadic scan (training side), sequential in t from
 * the end: the reference's DyadicScanFunction.backward branch at
 * src/mamba_integer_model.py:319-344, which computes the same quantities as
 * its Triton fast backward (src/triton_kernels/dyadic_scan.py:376-459):
 *   g[t] = grad_h[t] + decay[t] * g[t+1]   (decay = nums / 32768)
 *   grad_u[t] = (1 - decay[t]) * g[t]
 *   grad_nums[t] = (g[t] * (h[t-1] - u[t])) / 32768      (h[-1] = 0)
 * fp32, each operation rounded once, in that order.
 */
void orc_scan_convex_backward(const float* grad_h, const float* h, const float* u, const float* nums,
                              float* grad_u, float* grad_nums, int64_t Bsz, int64_t L, int64_t DN, int nthreads) {
#pragma omp parallel for collapse(2) schedule(static) ORC_THREADS(nthreads)
    for (int64_t b = 0; b < Bsz; b++)
        for (int64_t c = 0; c < DN; c++) {
            float acc = 0.0f;
            for (int64_t t = L - 1; t >= 0; t--) {
                const int64_t o = (b * L + t) * DN + c;
                const float d = nums[o] / 32768.0f;
                const float da = d * acc;
                acc = grad_h[o] + da;
                const float iw = 1.0f - d;
                grad_u[o] = iw * acc;
                const float hp = t > 0 ? h[o - DN] : 0.0f;
                const float diff = hp - u[o];
                const float gd = acc * diff;
                grad_nums[o] = gd / 32768.0f;
            }
        }
}

/*
 * Straight-through backward of the activation quantisation (training side),
 * src/triton_kernels/bitnet_kernels.py:77-95: per row with saved scale
 * amax[t] (the row's max |x|),
 *   grad_x = clamp((grad_xq * 127) / clamp(amax, min=0.01), -100, 100).
 */
void orc_quant_ste_backward(const float* grad_xq, const float* amax, float* grad_x, int64_t T, int64_t K) {
    for (int64_t t = 0; t < T; t++) {
        const float s = amax[t] != amax[t] ? amax[t] : (amax[t] < 0.01f ? 0.01f : amax[t]);
        for (int64_t k = 0; k < K; k++) {
            const float g = grad_xq[t * K + k] * 127.0f;
            grad_x[t * K + k] = clamp_t(g / s, -100.0f, 100.0f);
        }
    }
}

/*
 * The selective-scan section of MambaIntegerBlock.forward
 * (src/mamba_integer_model.py:419-444) from the dt_proj output onward:
 *   mod  = ste_clamp(dt_proj_out, -20, 20)                        (:422)
 *   nums = ste_clamp(base_decay_nums[d,n] + mod, 0, 32000)         (:424)
 *   dtv  = ste_clamp(squareplus(mod) * 0.01, 0.001, 0.1)           (:427)
 *   u    = (x * dtv) * B[n]                                         (:428)
 *   h    = convex dyadic scan (:436, :301-315)
 *   y    = sum_n h[n] * C[n], fused multiply-add n = 0..N-1         (:440)
 *   out  = y * sigmoid_alg(z)                                       (:444)
 * xact: [Bsz*L, D]; bc: rows of [B(N) | C(N)] at stride ldbc; modraw: [Bsz*L, D];
 * z: row stride ldz; base: [D, N]; out: [Bsz*L, D].
 * h_last (optional): final state [Bsz, D, N].
 */
void orc_ssm(const float* xact, const float* bc, int64_t ldbc, const float* modraw,
             const float* z, int64_t ldz, const float* base, int64_t Bsz, int64_t L, int64_t D,
             int64_t N, float* out, float* h_last, int nthreads) {
#pragma omp parallel for collapse(2) schedule(static) ORC_THREADS(nthreads)
    for (int64_t b = 0; b < Bsz; b++)
        for (int64_t d = 0; d < D; d++) {
            float h[64];
            for (int64_t n = 0; n < N; n++) h[n] = 0.0f;
            for (int64_t t = 0; t < L; t++) {
                int64_t row = b * L + t;
                float mod = ste_clamp(modraw[row * D + d], -20.0f, 20.0f);
                float dtv = ste_clamp(squareplus(mod) * 0.01f, 0.001f, 0.1f);
                float xdt = xact[row * D + d] * dtv;
                const float* Bv = bc + row * ldbc;
                const float* Cv = Bv + N;
                float y = 0.0f;
                for (int64_t n = 0; n < N; n++) {
                    float num = ste_clamp(base[d * N + n] + mod, 0.0f, 32000.0f);
                    float dec = num / 32768.0f;
                    float u = xdt * Bv[n];
                    float a = h[n] * dec;
                    float om = 1.0f - dec;
                    h[n] = a + om * u;
                }
                for (int64_t n = 0; n < N; n++) y = fmaf(h[n], Cv[n], y);
                out[row * D + d] = sigmoid_gate(y, z[row * ldz + d]);
            }
            if (h_last)
                for (int64_t n = 0; n < N; n++) h_last[(b * D + d) * N + n] = h[n];
        }
}

/* residual + out * res_gate (src/mamba_integer_model.py:447). */
void orc_residual(const float* res, const float* out, float g, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = res[i] + out[i] * g;
}

/* logits * output_scale (src/mamba_integer_model.py:494). */
void orc_scale(float* x, int64_t n, float s) {
    for (int64_t i = 0; i < n; i++) x[i] = x[i] * s;
}

/*
 * Integer dyadic selective scan (north_star form; state update as in
 * src/cuda_kernels/dyadic_mamba_kernel.cu:35-63 and
 * tests/test_mamba_scan.py:45-67, extended with the B/C terms):
 *   h[b,d,j] <- ((int64)h * n[d,j]) >> k  +  B[b,t,j] * x[b,t,d]
 *   y[b,t,d]  = sum_j C[b,t,j] * h[b,d,j]            (int64)
 * The shift is an arithmetic (flooring) right shift of the 64-bit product.
 * h is an int32 state: a value outside int32 is an overflow error.
 * x: [Bsz, L, D]; B, C: [Bsz, L, N]; n: [D, N]; h_io: [Bsz, D, N]; y: [Bsz, L, D].
 */
int orc_scan_i32(const int32_t* x, const int32_t* Bm, const int32_t* Cm, const int32_t* n, int k,
                 int64_t* y, int32_t* h_io, int64_t Bsz, int64_t L, int64_t D, int64_t N,
                 int nthreads) {
    if (N > 64 || k < 0 || k > 62) return ORC_ERR_INVALID;
    int err = 0;
#pragma omp parallel for collapse(2) schedule(static) ORC_THREADS(nthreads) reduction(| : err)
    for (int64_t b = 0; b < Bsz; b++)
        for (int64_t d = 0; d < D; d++) {
            int32_t h[64];
            for (int64_t j = 0; j < N; j++) h[j] = h_io[(b * D + d) * N + j];
            for (int64_t t = 0; t < L; t++) {
                int64_t xv = x[(b * L + t) * D + d];
                const int32_t* Bv = Bm + (b * L + t) * N;
                const int32_t* Cv = Cm + (b * L + t) * N;
                int64_t acc = 0;
                for (int64_t j = 0; j < N; j++) {
                    int64_t p = (int64_t)h[j] * (int64_t)n[d * N + j];
                    int64_t hn = (p >> k) + (int64_t)Bv[j] * xv;
                    if (hn > INT32_MAX || hn < INT32_MIN) err = 1;
                    h[j] = (int32_t)hn;
                    acc += (int64_t)Cv[j] * (int64_t)h[j];
                }
                y[(b * L + t) * D + d] = acc;
            }
            for (int64_t j = 0; j < N; j++) h_io[(b * D + d) * N + j] = h[j];
        }
    return err ? ORC_ERR_OVERFLOW : ORC_OK;
}
