/*
 * mi_b200.h -- C ABI of the B200 (sm_100a) Mamba-Integer hot path.
 *
 * Conventions (all entry points):
 *   - every buffer is caller-owned device memory (the library never allocates
 *     or frees, except where an entry point says so);
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     work is enqueued on it with no host synchronisation;
 *   - the return value is a status code: MI_OK (0) or a negative MI_ERR_*;
 *     argument/shape errors are detected on the host before any launch;
 *   - device-side conditions (integer overflow, a bounded wait that expired)
 *     are recorded in a per-device error word read by mi_device_error().
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the reference repository).
 */
#ifndef MI_B200_H
#define MI_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MI_OK 0
#define MI_ERR_INVALID (-1)     /* bad pointer, size or stride */
#define MI_ERR_UNSUPPORTED (-2) /* shape/config this build does not handle */
#define MI_ERR_CUDA (-3)        /* CUDA runtime / driver error at launch */
#define MI_ERR_DEVICE (-4)      /* device error word was set (see mi_device_error) */

/* device error word bits */
#define MI_DEV_OVERFLOW 0x1     /* integer scan: a state or output left int32 */
#define MI_DEV_TIMEOUT 0x2      /* a bounded mbarrier wait expired */
#define MI_DEV_PRECOND 0x4      /* an input outside the kernel's stated range */

int mi_version(void);
const char* mi_status_string(int status);

/* Reads (and clears, if `clear`) the device error word of the current device.
 * Synchronises `stream`. */
int mi_device_error(int* out, int clear, void* stream);

/*
 * Integer dyadic selective scan.
 *   h[b,d,j] <- ((int64)h * n[d,j]) >> k  +  B[b,t,j] * x[b,t,d]
 *   y[b,t,d]  = sum_j C[b,t,j] * h[b,d,j]
 * x [batch,L,D], B/C [batch,L,N], n [D,N], h_io [batch,D,N] (initial state
 * in, final state out), y [batch,L,D] int32 (y32) or int64 (y64): exactly one
 * of y32 / y64 is non-NULL.  Preconditions checked on the device (error word
 * MI_DEV_PRECOND): 0 <= n <= 2^k; |x|, |B|, |C| <= 32767.  A state that
 * leaves int32, or a y32 value that does, sets MI_DEV_OVERFLOW.
 * Supports N = 16; 1 <= k <= 30; D % 4 == 0; every pointer 16-byte aligned.
 * Replaces: launch_dyadic_scan, src/cuda_kernels/dyadic_mamba_kernel.cu:135-153
 * (state update :53-59), extended with the B/C terms of the selective scan.
 */
int mi_scan_i32(const int32_t* x, const int32_t* B, const int32_t* C, const int32_t* n, int k,
                int32_t* y32, int64_t* y64, int32_t* h_io, int batch, int L, int D, int N,
                void* stream);

/*
 * BitShiftNorm forward (CPU-path semantics): centre (twice: BitShiftNorm.forward
 * then BitShiftNormFunction.forward; once if center_once), var = mean(xc^2),
 * power-of-2 scale s from the threshold table, y = ((xc*s)*gamma)*step.
 * x, y [T,D]; gamma [D]; step [1] (device); inv_rms [T] (may be NULL).
 * D % 32 == 0, 32 <= D <= 1024.
 * Replaces: fast_bitshift_norm, src/triton_kernels/bitnet_kernels.py:295
 * (and launch_bitshift_norm, src/cuda_kernels/bitshift_norm.cu:97-114).
 */
int mi_bitshift_norm(const float* x, const float* gamma, const float* step, float* y, float* inv_rms,
                     int T, int D, int center_once, void* stream);

/*
 * Per-token absmax int8 quantisation (activation_quant_dynamic):
 *   s = max(amax|x|, 1e-8); xq = clamp(rne(x * (127 * (1/s))), +-127);
 *   xscale = s / 127.
 * x [T, >=K] row stride ldx; xq [T, >=K] row stride ldq (int8).
 * amax (optional, [T]): max|x| of each row already computed by the producer
 * of x (NULL: computed here).  clear (optional, [T]): set to 0 by this call,
 * row for row -- the row-maximum array of a kernel that follows and
 * accumulates by atomicMax (the fused scan), without a separate fill.
 * Replaces: fast_quantize_activations, src/triton_kernels/bitnet_kernels.py:98.
 */
int mi_quantize_rows(const float* x, int ldx, int T, int K, int8_t* xq, int ldq, float* xscale,
                     const float* amax, float* clear, void* stream);

/*
 * Row pre-pass in front of a BitLinear: optional residual update, BitShiftNorm,
 * int8 quantisation, in one pass over each row.
 *   source row r = ids ? emb[ids[t]] : x[t] (+ delta[t] * (*res_gate) if delta)
 *   (an id outside [0, vocab) reads a zero row and sets MI_DEV_PRECOND)
 *   x_out[t] = r (if x_out; the new residual stream)
 *   y = BitShiftNorm(r); (y_norm[t] = y if y_norm)
 *   (xq[t], xscale[t]) = quantise(y)
 * D % 32 == 0, 32 <= D <= 1024.
 * Replaces the sequence BitShiftNorm -> activation_quant_dynamic in
 * src/mamba_integer_model.py:397-400 / :447 -> :398 / :492-494.
 */
int mi_rowprep(const float* x, const float* delta, const float* res_gate, const int64_t* ids,
               const float* emb, int vocab, float* x_out, const float* gamma, const float* step, float* y_norm,
               int8_t* xq, float* xscale, int T, int D, void* stream);

/* BitLinear epilogues */
#define MI_EPI_I32 0        /* out int32 [M,N]: the raw accumulators */
#define MI_EPI_F32_SCALED 1 /* out fp32: acc * (w_scale * a_scale[m]) [* out_scale] */

/*
 * Ternary BitLinear contraction on tcgen05 (kind::i8, int32 accumulators in
 * TMEM).  A int8 [M,K] (row stride lda), W int8 ternary [N,K] (dense rows),
 * out [M,N] row stride ldo.  a_scale [M], w_scale [1], out_scale [1] are
 * device pointers (out_scale may be NULL).  K % 16 == 0, lda % 16 == 0,
 * N % 16 == 0.
 * Replaces: launch_bitlinear, src/cuda_kernels/bitlinear.cu:74-90, and the
 * matmul + rescale of BitLinear.forward, src/rational_bitnet.py:204-208.
 */
int mi_bitlinear_i8(const int8_t* A, int lda, const int8_t* W, const float* a_scale,
                    const float* w_scale, const float* out_scale, void* out, int ldo, int M, int N,
                    int K, int epilogue, void* stream);

/*
 * 2-bit packed ternary weights.  Wp [N, K/4] bytes, row-major; each
 * little-endian 32-bit word holds 16 consecutive weights k = 16g .. 16g+15,
 * weight 16g + 4q + j in bits [p, p + 2), p = 4j + 2(q & 1) + 16(q >> 1), as a
 * 2-bit two's complement value (00 = 0, 01 = +1, 11 = -1).
 * mi_pack_ternary: W int8 [N, K] (row stride ldw) -> Wp; K % 16 == 0,
 * ldw % 16 == 0; a value outside {-1, 0, 1} is stored as 0 and sets
 * MI_DEV_PRECOND.
 * Replaces the ternarisation result of weight_quant_ternary,
 * src/rational_bitnet.py:63-85 (kept as fp32 {-1,0,1} by the reference and
 * as int8 by scripts/export_int8.py:77-81): the packed form is this library's
 * storage format.
 */
int mi_pack_ternary(const int8_t* W, int ldw, uint8_t* Wp, int N, int K, void* stream);

/*
 * mi_bitlinear_i8 with 2-bit packed weights: the TMA loads packed K-slices,
 * the kernel expands them to int8 in shared memory and feeds the same
 * tcgen05 kind::i8 MMAs; results are identical to mi_bitlinear_i8 on the
 * unpacked weights.  K % 64 == 0 (packed rows of K/4 bytes, 16-byte pitch).
 * Replaces: launch_bitlinear, src/cuda_kernels/bitlinear.cu:74-90, and the
 * matmul + rescale of BitLinear.forward, src/rational_bitnet.py:204-208.
 */
int mi_bitlinear_packed(const int8_t* A, int lda, const uint8_t* Wp, const float* a_scale,
                        const float* w_scale, const float* out_scale, void* out, int ldo, int M,
                        int N, int K, int epilogue, void* stream);

/*
 * BitLinear with the BitShift-norm + squareplus epilogue of BASELINE config 3
 * (2-bit packed ternary weights).  acc [M, N] int32 (row stride ldc) receives
 * the exact accumulators; out [M, N] fp32 (row stride ldo) receives, per row,
 *   y = acc * (w_scale * a_scale[m]);  BitShiftNorm of y with the mean and the
 *   power-of-two variance scale taken exactly from the integer row sums
 *   S1 = sum acc, S2 = sum acc^2;  o = ((y - mean) * s * gamma[n]) * step;
 *   out = squareplus(ste_clamp(o, -50, 50)).
 * (The reference has no fused GEMM + norm: this chains its stages, and
 * defines the statistics from exact integers so that they do not depend on
 * a summation order; the restatement is oracle/mi_oracle.c:orc_bitlinear_norm_sqp.)
 * gamma [N] and step [1] are device pointers.  stats_ws: caller workspace of
 * 2*M uint64 (S1, S2 per row, zeroed by the call).  K % 64 == 0,
 * N % 16 == 0, N*K <= 2^24; acc, out, gamma 16-byte aligned.
 * Replaces the chain BitLinear.forward (src/rational_bitnet.py:204-208) ->
 * BitShiftNorm (src/mamba_integer_model.py:199-222) -> fused_squareplus_clamp
 * (src/triton_kernels/fused_activations.py:229) on one row of outputs.
 */
int mi_bitlinear_packed_norm_sqp(const int8_t* A, int lda, const uint8_t* Wp, const float* a_scale,
                                 const float* w_scale, const float* gamma, const float* step, int32_t* acc,
                                 int ldc, float* out, int ldo, uint64_t* stats_ws, int M, int N, int K,
                                 void* stream);

/*
 * Causal depthwise conv (4 taps, bias first then one FMA per tap) +
 * ste_clamp(-50, 50) + squareplus (3 Newton steps), then int8 quantisation of
 * each row of the activation.
 * xz rows [batch*L] with stride ldx: the first D columns are the conv input;
 * w [D,4], bias [D]; act [batch*L, D]; xq [batch*L, D]; xscale [batch*L];
 * amax_ws: caller-provided workspace of batch*L floats (required with xq).
 * Replaces: conv1d + fused_squareplus_clamp, src/mamba_integer_model.py:404-411
 * (fused_squareplus_clamp: src/triton_kernels/fused_activations.py:229).
 */
int mi_conv_act_quant(const float* xz, int ldx, const float* w, const float* bias, float* act,
                      int8_t* xq, float* xscale, float* amax_ws, int batch, int L, int D, void* stream);

/*
 * mi_conv_act_quant in one kernel and without a workspace: each CTA owns whole
 * rows (D/4 threads, 4 channels each) for a chunk of positions, reduces the
 * row absmax in the block and quantises from registers.  Same results as
 * mi_conv_act_quant.  D % 4 == 0, D <= 4096; xq required.
 * Replaces: conv1d + fused_squareplus_clamp + activation_quant_dynamic,
 * src/mamba_integer_model.py:404-411 (quantisation: src/rational_bitnet.py:102-111).
 */
int mi_conv_act_quant_rows(const float* xz, int ldx, const float* w, const float* bias, float* act,
                           int8_t* xq, float* xscale, int batch, int L, int D, void* stream);

/*
 * mi_conv_act_quant without the caller-provided workspace, for hosts that
 * cannot call cudaMalloc (a runtime whose device memory belongs to another
 * allocator, a serving loop that must not allocate).  No counterpart in the
 * reference.  The row-absmax scratch is a fixed array inside the library:
 * batch * L <= 262144 rows, larger requests return MI_ERR_UNSUPPORTED.  xq and
 * xscale are required (this variant always quantises).  The first call on a
 * device looks the array's device address up and keeps it for the life of the
 * process (make that first call before any stream capture; do not call it on a
 * device after cudaDeviceReset there).  Every call shares the array: calls that
 * overlap on the GPU race with each other; each call zero-fills the rows it
 * uses before using them.  Allocates nothing.
 */
int mi_conv_act_quant_noalloc(const float* xz, int ldx, const float* w, const float* bias, float* act,
                              int8_t* xq, float* xscale, int batch, int L, int D, void* stream);

/*
 * Selective-scan section of MambaIntegerBlock from the dt_proj output on:
 * decay clamp, dt, u = (x*dt)*B, convex dyadic scan h = h*d + (1-d)*u with
 * d = n/2^15, y = sum_n h*C (FMA, n ascending), gate y*sigmoid_alg(z).
 * act [batch*L, D]; bc rows (stride ldbc): B at [0,N), C at [N,2N);
 * modraw [batch*L, D]; z rows stride ldz; base [D,N]; y [batch*L, D].
 * amax (optional, [batch*L], zero on entry) receives max|y| per row (feed it
 * to mi_quantize_rows; the quantisation of the dt rows that precedes the scan
 * can clear it).
 * N == 16.  Results are the reference's bits; the one exception is the sign
 * of a zero: where B holds -0.0 (the model's x_proj output never does), a
 * state the reference leaves at -0.0 may come out +0.0.
 * Replaces: DyadicScanFunction.apply / dyadic_scan_triton_fast
 * (src/mamba_integer_model.py:419-444, src/triton_kernels/dyadic_scan.py:462).
 */
int mi_ssm_scan(const float* act, const float* bc, int ldbc, const float* modraw, const float* z,
                int ldz, const float* base, float* y, float* amax, int batch, int L, int D, int N,
                void* stream);

/*
 * mi_ssm_scan with the dt_proj BitLinear fused in: instead of the dt_proj
 * output, takes the int8-quantised dt rows dtq [batch*L, ldq] (R values used,
 * ldq % 16 == 0), their scales dts [batch*L], the ternary dt_proj weights
 * w_dt int8 [D, ceil16(R)] (zero-padded) and w_dt_scale [1]; each channel
 * forms the exact int32 dot product and the BitLinear rescale
 * acc * (w_dt_scale * dts[t]) itself.  R <= 64.
 * split = kernel variant: 1, 2, 4 or 8 lanes per channel, or 3 = one lane per
 * channel with each chunk's phases pipelined over four warps (two staging
 * and decay, recurrence, gate); 0 = automatic (3 from 64 positions on, where
 * it measured fastest at every batch; 1 for shorter sequences).  All variants
 * give identical results.
 * h_out (optional, [batch, D, N], 16-byte aligned) receives the states after
 * the last position (the starting point of mi_ssm_step).  The sign-of-zero
 * note of mi_ssm_scan applies.
 * Replaces: dt_proj + DyadicScanFunction section, src/mamba_integer_model.py:419-444
 * (BitLinear rescale: src/rational_bitnet.py:204-208).
 */
int mi_ssm_scan_dt(const float* act, const float* bc, int ldbc, const int8_t* dtq, int ldq,
                   const float* dts, const int8_t* w_dt, const float* w_dt_scale, int R,
                   const float* z, int ldz, const float* base, float* y, float* amax, float* h_out,
                   int batch, int L, int D, int N, int split, void* stream);

/*
 * Decode: one new position for `batch` independent streams (one CTA per
 * stream).  The reference has no step API; it recomputes
 * MambaIntegerModel.forward over the whole sequence for every token
 * (scripts/inference.py:148-160).  These steps give the bits that forward
 * gives the last position: same operations, same order.
 *
 * mi_conv_step: x_t = first D columns of xz row b (row stride ldx); win
 * [batch, 3, D] holds x_{t-3}, x_{t-2}, x_{t-1} and is advanced in place;
 * act (optional) [batch, D] = squareplus(ste_clamp(conv, +-50)); xq [batch, D]
 * int8 and xscale [batch] its quantisation.  D % 4 == 0, D <= 4096.
 * Replaces: conv1d + fused_squareplus_clamp at the last position,
 * src/mamba_integer_model.py:404-411 (and launch_conv1d_step,
 * src/cuda_kernels/conv1d_step.cu:61-78, whose bias-last order differs).
 */
int mi_conv_step(const float* xz, int ldx, const float* w, const float* bias, float* win, float* act,
                 int8_t* xq, float* xscale, int batch, int D, void* stream);

/*
 * mi_ssm_step: xp row b (stride ldxp) = [dt (R) | B (N) | C (N)], the x_proj
 * output; the dt row is quantised (activation_quant_dynamic), dt_proj is the
 * exact int32 dot product with w_dt int8 [D, R16] and its rescale, then
 * decay / dt / u, one convex update of h [batch, D, N] (in place), y = sum h*C,
 * the gate with z (row stride ldz); y (optional) [batch, D] and its int8
 * quantisation xq [batch, D], xscale [batch].  N == 16, D <= 4096, R <= 64.
 * Replaces: the dt_proj + DyadicScanFunction section at the last position,
 * src/mamba_integer_model.py:419-444.
 */
int mi_ssm_step(const float* act, const float* xp, int ldxp, int R, const int8_t* w_dt,
                const float* w_dt_scale, const float* z, int ldz, const float* base, float* h, float* y,
                int8_t* xq, float* xscale, int batch, int D, int N, void* stream);

/*
 * mi_decode_mid: mi_conv_step, the x_proj BitLinear and mi_ssm_step in one
 * kernel (one CTA per stream): everything between a layer's in_proj and
 * out_proj GEMMs for one decode position.  xz [batch, ldx] = [x (D) | z (D)]
 * (the in_proj output); win [batch, 3, D] and h [batch, D, N] advanced in
 * place; w_x int8 [R + 2N, D] with its scale w_x_scale [1] (x_proj as exact
 * int32 dot products, rescaled as the GEMM epilogue does); w_dt int8
 * [D, R16], base [D, N]; xp_out (optional) [batch, R + 2N] receives the
 * x_proj output; xq [batch, D] / xscale [batch]: y quantised for out_proj.
 * N == 16, D % 16 == 0, D <= 4096, R <= 64.
 * Replaces: the conv .. gate section of MambaIntegerBlock.forward at the last
 * position, src/mamba_integer_model.py:404-444.
 */
int mi_decode_mid(const float* xz, int ldx, const float* conv_w, const float* conv_b, float* win,
                  const int8_t* w_x, const float* w_x_scale, int R, const int8_t* w_dt,
                  const float* w_dt_scale, const float* base, float* h, float* xp_out, int8_t* xq,
                  float* xscale, int batch, int D, int N, void* stream);

/*
 * mi_decode_mid_packed: mi_decode_mid with the x_proj weights in the 2-bit
 * packed form of mi_pack_ternary (w_x_packed uint8 [R + 2N, D/4], 4-byte
 * aligned), which every stream reads a quarter as many bytes of.  Same
 * results bit for bit.  D % 64 == 0 (a cluster of 4 CTAs per stream, each a
 * slice of whole 16-weight words), D <= 4096, R <= 64, N == 16.
 * Replaces: as mi_decode_mid, src/mamba_integer_model.py:404-444.
 */
int mi_decode_mid_packed(const float* xz, int ldx, const float* conv_w, const float* conv_b, float* win,
                         const uint8_t* w_x_packed, const float* w_x_scale, int R, const int8_t* w_dt,
                         const float* w_dt_scale, const float* base, float* h, float* xp_out, int8_t* xq,
                         float* xscale, int batch, int D, int N, void* stream);

/*
 * mi_argmax_rows: out[t] = torch.argmax(x[t, :V]) (first index of the
 * maximum; NaN counts as the maximum), x rows of stride ldx.
 * Replaces the greedy choice over logits[:, -1, :] in the generation loop,
 * scripts/inference.py:150-158 (which samples with temperature 0.8).
 */
int mi_argmax_rows(const float* x, int ldx, int T, int V, int64_t* out, void* stream);

/* Convex dyadic scan on materialised inputs: h = h*(n/2^15) + (1-n/2^15)*u.
 * u, nums, h [batch, L, DN].
 * Replaces: dyadic_scan_triton_fast(u, nums), src/triton_kernels/dyadic_scan.py:462. */
int mi_scan_convex(const float* u, const float* nums, float* h, int batch, int L, int DN, void* stream);

/*
 * Training side.  Backward of the convex dyadic scan: grad_h, h (the forward's
 * output), u, nums [batch, L, DN] fp32 -> grad_u, grad_nums (same shape):
 *   g[t] = grad_h[t] + (nums[t]/32768) * g[t+1];  grad_u = (1 - nums/32768) * g;
 *   grad_nums[t] = (g[t] * (h[t-1] - u[t])) / 32768  (h[-1] = 0).
 * Replaces: dyadic_scan_backward_triton_fast, src/triton_kernels/dyadic_scan.py:376-459
 * (DyadicScanFunction.backward, src/mamba_integer_model.py:316-344).
 */
int mi_scan_convex_backward(const float* grad_h, const float* h, const float* u, const float* nums,
                            float* grad_u, float* grad_nums, int batch, int L, int DN, void* stream);

/*
 * Training side.  Straight-through backward of the per-token int8 activation
 * quantisation: grad_xq [T, K], amax [T] (each row's max |x|, the scale the
 * forward saved) -> grad_x [T, K] =
 *   clamp((grad_xq * 127) / clamp(amax, min=0.01), -100, 100).
 * With K % 4 == 0, grad_xq and grad_x must be 16-byte aligned.
 * Replaces: QuantizeActivationsFunction.backward, src/triton_kernels/bitnet_kernels.py:77-95.
 */
int mi_quant_ste_backward(const float* grad_xq, const float* amax, float* grad_x, int T, int K, void* stream);

/* Element-wise ops (n elements, contiguous).
 * Replace fused_squareplus_clamp / fused_ste_clamp / fused_sigmoid_gate,
 * src/triton_kernels/fused_activations.py:229, :511, :399. */
int mi_squareplus_clamp(const float* x, float* y, int64_t n, float lo, float hi, void* stream);
int mi_ste_clamp(const float* x, float* y, int64_t n, float lo, float hi, void* stream);
int mi_sigmoid_gate(const float* y, const float* z, float* out, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MI_B200_H */
