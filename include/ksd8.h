/*
 * ksd8.h — C ABI of the B200 (sm_100a) INT8 hot path of KSDraft.
 *
 * Every entry point takes raw device pointers, sizes and row strides (in
 * elements), a `status` word in device memory (may be NULL) that kernels use
 * to report device-side failures (timeouts), and a cudaStream_t passed as
 * `void*` (NULL = legacy default stream).  Work is only enqueued on that
 * stream: nothing synchronises, nothing allocates device memory.  The return
 * value is a KSD8_* status: argument errors are detected on the host before
 * any launch.
 *
 * Layout conventions follow the reference int8 tier (ksdraft/kernels/quant.py:1-14):
 * row-major, the quantised dimension is the LAST one, weights are (N, K),
 * scales are fp16, one per 128 consecutive elements, codes in [-127, 127].
 *
 * Reference interfaces replaced (paths within curvedinf/ksdraft):
 *   ksd8_quantize_rows        ksdraft/kernels/quant.py:30 quantize_last_dim,
 *                             ksdraft/train/stages.py:27 quantize_last_dim_dithered
 *   ksd8_quantize_cols        quantize_last_dim(t.t().contiguous()) and
 *                             quantize_last_dim(dequantize_last_dim(c, s).t()),
 *                             ksdraft/kernels/ks3_int8.py:350,407-424
 *   ksd8_w8a8_gemm            ksdraft/kernels/gemm.py:53 w8a8_gemm (+ the _w8a8_gemm_kernel at :18)
 *   ksd8_w8a8_group_partials  per-group int32 dot products of gemm.py:34-45 (parity probe)
 *   ksd8_ks3_pack             ksdraft/kernels/ks3_int8.py:262-277 _repack_masters (spine + warp part),
 *                             :87 pack_spine, :158 _warp_scalars
 *   ksd8_ks3_spine_quant      ksdraft/kernels/ks3_int8.py:169-234 _spine_features followed by
 *                             quantize_last_dim(h) (:284, :331)
 *   ksd8_ks3_spine_table      the (chart, LUT index)-only part of ks3_int8.py:206-227
 *   ksd8_ks3_vjp              ksdraft/kernels/ks3_int8.py:354-410 (geometry VJP, dc, its two quantisations)
 *   ksd8_ks3_vjp_reduce       ksdraft/kernels/ks3_int8.py:381-395 (column reductions, STE factors)
 *   ksd8_ks3_vjp_reduce_f32   the same, fp32 outputs (handoff values for the masters' grads)
 *   ksd8_rosa_pack_bits       ksdraft/model/rosa.py:156-158 (bits = proj > 0) and the int8 bit inputs
 *                             of rosa.py:40 _match_payload_sign
 *   ksd8_rosa_match           ksdraft/model/rosa.py:40-98 _match_payload_sign (+ payload multiply of :164)
 *   ksd8_rosa_match_scratch   the same, adaptive matcher with caller scratch
 *   ksd8_rosa_payload_bwd     the payload gradient of rosa.py:164 through the Int8Linear STE of
 *                             out_proj (ksdraft/kernels/linear.py:88-94, incl. the scale term)
 *   ksd8_rosa_timemix_quantize ksdraft/model/rosa.py:128-133 _shifted followed by the per-token
 *                             quantisation of Int8Linear.forward (ksdraft/kernels/linear.py:69)
 *   ksd8_adamw_step           torch.optim.AdamW.step over fp32 masters (ksdraft/train/__init__.py:166)
 *   ksd8_adamw_step_scaled    the same after gradient clipping (ksdraft/train/__init__.py:165)
 *   ksd8_adamw_multi          the same over several tensors in one launch
 *   ksd8_grad_clip_coef       torch.nn.utils.clip_grad_norm_ norm and coefficient (:165)
 *   ksd8_fp16_tanh_table      the fp16 torch.tanh of ksdraft/kernels/ks3_int8.py:366-367 (parity probe)
 *   ksd8_dspine_ln_fwd        ksdraft/model/spine.py:64-69 AdjacentInjection.forward (gate and
 *                             injection combine around the low-rank GEMMs) followed by the
 *                             block's ln_ffn (ksdraft/model/block.py:41)
 *   ksd8_dspine_ln_bwd        the autograd backward of the same (LayerNorm, sigmoid gate)
 *   ksd8_transfer_rows        ksdraft/train/__init__.py:80-84, the transfer-space term per token
 *   ksd8_transfer_bwd         its gradient (the F.normalize backward) for a loss coefficient
 *   ksd8_rosa_decode_build    no reference counterpart: the sorted key run behind
 *                             ksd8_rosa_decode_step, built from a context's k bits
 *   ksd8_rosa_decode_merge    no reference counterpart: the same run, grown by merging the
 *                             keys appended since it was built
 *   ksd8_rosa_decode_step     ksdraft/model/rosa.py:40-98 _match_payload_sign (+ :164 payload)
 *                             answered for positions appended to a matched context
 *   ksd8_rosa_credits         ksdraft/kernels/rosa_credit_gpu.py:25-48 _chunk_credits
 */
#ifndef KSD8_H_
#define KSD8_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define KSD8_OK 0
#define KSD8_ERR_SHAPE 1          /* inconsistent sizes (reference: ValueError) */
#define KSD8_ERR_ALIGN 2          /* pointer / stride not aligned as required */
#define KSD8_ERR_DTYPE 3          /* unsupported dtype code (reference: TypeError) */
#define KSD8_ERR_LAUNCH 4         /* CUDA launch / driver error */
#define KSD8_ERR_DEVICE_TIMEOUT 5 /* a bounded device-side wait gave up */
#define KSD8_ERR_UNSUPPORTED 6    /* valid request outside this build (e.g. group != 128 on the GEMM) */
#define KSD8_ERR_ARG 7            /* bad scalar argument */
#define KSD8_ERR_NONFINITE 8      /* status bit: an fp16 output overflowed (FP16 handoff) */

/* ---- dtype codes ---- */
#define KSD8_F32 0
#define KSD8_F16 1
#define KSD8_BF16 2
#define KSD8_I8 3

/* ---- quantiser flags ---- */
#define KSD8_Q_ROUND_F16 1   /* round the input through fp16 first (x.float().to(float16)) */
#define KSD8_Q_DITHER 2      /* add PTQR rounding dither from the Philox4x32-10 counter RNG */
#define KSD8_Q_RELU 4        /* not used by the reference path; reserved */
#define KSD8_Q_PLAIN_LOADS 8 /* use the thread-load kernels instead of the bulk/TMA-staged
                                ones (identical results; the staged kernels need 16-byte
                                aligned rows and are chosen by default when they apply) */

/* ---- GEMM epilogue flags ---- */
#define KSD8_EPI_CLAMP_F16 1  /* fp16 output: saturate +-inf to +-65504 (ks3_int8.py:241-242) */
#define KSD8_EPI_BIAS 2       /* add fp32 bias[n] after the group sum (linear.py:71) */
#define KSD8_EPI_FLAG_NONFINITE 4 /* fp16 output or ROUND_F16: set KSD8_ERR_NONFINITE in *status on inf/nan */
#define KSD8_EPI_ROUND_F16 8  /* fp32 output holds float(fp16(y)): the FP16 grad handoff of
                                 ks3_int8.py:75-84 written straight into an fp32 grad buffer */
#define KSD8_EPI_IF_STATUS 16 /* predicated launch: the kernel returns at once unless *status
                                 is non-zero (the handoff's fp32 overflow fallback, decided on
                                 the device without a host round trip) */

/* ---- nonlinear modes of the KS3 cell (ks3_int8.py:22-28) ---- */
#define KSD8_NL_FP32 0
#define KSD8_NL_FP16 1
#define KSD8_NL_INT8 2

int ksd8_version(void);
/* SMs per device that the persistent kernels (GEMM, VJP) leave free, for
 * collectives running at the same time (e.g. NCCL capped to that many CTAs):
 * their grids shrink to sm_count - n.  Process-wide, 0 by default. */
int ksd8_set_sm_reserve(int n);
int ksd8_get_sm_reserve(void);
const char* ksd8_status_string(int status);
/* Last CUDA runtime error seen by a launch in this thread (cudaError_t as int). */
int ksd8_last_cuda_error(void);
int ksd8_sm_count(int device);

/* Quantise `rows` rows of `k` elements (row stride ldx) in groups of `group`
 * along the row.  codes: (rows, k) row stride ldc (padded lanes are not
 * written); scales: (rows, ceil(k/group)) fp16, contiguous.  With
 * KSD8_Q_DITHER, code = round(x/scale + (U - 0.5) * 2 * dither), U =
 * (philox(seed, offset + flat_index) >> 8) * 2^-24, flat_index = row * Kp + col
 * over the padded (rows, Kp) grid. */
int ksd8_quantize_rows(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t ldx,
                       int group, int flags, float dither, uint64_t seed, uint64_t offset,
                       int8_t* codes, int64_t ldc, void* scales, int* status, void* stream);

/* Transposed quantisation: x is (rows, cols) with row stride ldx.  The output
 * is x^T (cols, rows) quantised along `rows` in groups of `group`:
 * codes_t (cols, rows) row stride ldct, scales_t (cols, ceil(rows/group)).
 * When x_dtype == KSD8_I8, x holds int8 codes whose real value is
 * code * x_scales[r, c / x_group] (x_scales: (rows, ceil(cols/x_group)) fp16),
 * i.e. dequantize -> transpose -> requantize in one pass. */
int ksd8_quantize_cols(const void* x, int x_dtype, const void* x_scales, int x_group,
                       int64_t rows, int64_t cols, int64_t ldx, int group, int flags,
                       int8_t* codes_t, int64_t ldct, void* scales_t, int* status, void* stream);

/* Y(M,N) = sum_g float(A_g . W_g^T) * sa[m,g] * sw[n,g], int32 dot per
 * 128-wide K group on tcgen05 tensor cores, fp32 group sum in the canonical
 * order acc = fmaf(RN(float(dot_g) * sa[m,g]), sw[n,g], acc) for g = 0..G-1.
 * a: (m, k) int8, row stride k; w: (n, k) int8, row stride k; k % 128 == 0,
 * group must be 128; a_scales (m, k/128), w_scales (n, k/128) fp16.
 * out_dtype: KSD8_F32 / KSD8_F16 / KSD8_BF16, row stride ldo. */
int ksd8_w8a8_gemm(const int8_t* a, const void* a_scales, const int8_t* w, const void* w_scales,
                   int64_t m, int64_t n, int64_t k, int group, void* out, int out_dtype,
                   int64_t ldo, const float* bias, int epi_flags, int* status, void* stream);

/* Parity probe: the per-group int32 partial dot products of the same
 * tensor-core main loop, out (k/128, m, n) int32. */
int ksd8_w8a8_group_partials(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                             int32_t* out, int* status, void* stream);

/* KS3 pack of the small per-chart tensors from fp32 masters:
 * coefficients (charts*6) -> spine_codes (charts, 6) int8 + spine_scale (charts) fp16
 * (one GS group per 6-wide row, pack_spine); raw_scale/raw_shift (charts) ->
 * softplus(.)+1e-4 and 0.5*tanh(.) quantised per element (one group each)
 * into int8 codes + fp16 scales (the warp-scalar buffers of KS3Int8Cell). */
int ksd8_ks3_pack(const float* coefficients, const float* raw_scale, const float* raw_shift,
                  int64_t charts, int8_t* spine_codes, void* spine_scale,
                  int8_t* warp_scale_codes, void* warp_scale_scales, int8_t* warp_shift_codes,
                  void* warp_shift_scales, int* status, void* stream);

/* Composed KS3 spine on fp16 coordinates (M, charts) followed by GS128
 * requantisation of h along the charts: h_codes (M, charts), h_scales
 * (M, ceil(charts/128)).  The warp scalars are given as their int8 codes and
 * fp16 scales (one group per chart) and dequantised into the arithmetic
 * domain of the mode (fp32 for KSD8_NL_FP32, fp16 otherwise).  With
 * warp_*_codes == NULL the matching *_scales array holds the already
 * dequantised fp16 scalars (the interface of ks3_triton.py:159 project_fused).
 * lut: the 256-entry int8 tanh table (make_tanh_lut). */
int ksd8_ks3_spine_quant(const void* coords, int64_t m, int64_t charts,
                         const int8_t* spine_codes, const void* spine_scale,
                         const int8_t* warp_scale_codes, const void* warp_scale_scales,
                         const int8_t* warp_shift_codes, const void* warp_shift_scales,
                         const int8_t* lut, int nonlinear, const void* table, int8_t* h_codes,
                         void* h_scales, int* status, void* stream);

/* Per-chart table of the 'int8' spine term for the 256 LUT indices
 * (table (charts, 256) fp16, 16-byte aligned): everything of
 * ks3_int8.py:206-227 that depends only on (chart, index).  Passing it to
 * ksd8_ks3_spine_quant (KSD8_NL_INT8) selects the table-driven kernel, which
 * gives the same codes and scales. */
int ksd8_ks3_spine_table(int64_t charts, const int8_t* spine_codes, const void* spine_scale,
                         const int8_t* warp_scale_codes, const void* warp_scale_scales,
                         const int8_t* warp_shift_codes, const void* warp_shift_scales,
                         const int8_t* lut, void* table, int* status, void* stream);

/* KS3 geometry VJP (fp16 arithmetic as the reference) on value = fp16(g @ up)
 * and the saved fp16 coordinates, both (M, charts).  Writes dc quantised
 * along charts (dc_codes (M, charts), dc_scales (M, charts/128)) and along
 * tokens (dct_codes (charts, M), dct_scales (charts, ceil(M/128))), and
 * per-128-token-tile column partial sums partials (ceil(M/128), 8, charts) fp32
 * in the order d0..d5, dscale_t, dshift_t (dshift_t before its 0.5 factor).
 * charts must be a multiple of 128; value and coords 16-byte aligned (they
 * are read as TMA tiles).  A device-side wait that gives up sets
 * KSD8_ERR_DEVICE_TIMEOUT in *status (status may be NULL). */
int ksd8_ks3_vjp(const void* value, const void* coords, int64_t m, int64_t charts,
                 const int8_t* spine_codes, const void* spine_scale,
                 const int8_t* warp_scale_codes, const void* warp_scale_scales,
                 const int8_t* warp_shift_codes, const void* warp_shift_scales,
                 int8_t* dc_codes, void* dc_scales, int8_t* dct_codes, void* dct_scales,
                 float* partials, int* status, void* stream);

/* Reduce the VJP partials over token tiles (fixed order), round to fp16 and
 * apply the STE factors of ks3_int8.py:391-395: dcoeff (charts, 6),
 * dscale (charts), dshift (charts), all fp16.  Sets KSD8_ERR_NONFINITE in
 * *status when one of them is not finite (FP16 handoff check). */
int ksd8_ks3_vjp_reduce(const float* partials, int64_t n_tiles, int64_t charts,
                        const float* raw_scale, const float* raw_shift, void* dcoeff16,
                        void* dscale16, void* dshift16, int* status, void* stream);

/* ksd8_ks3_vjp_reduce with fp32 outputs holding float(fp16 value): the
 * gradients as the fp32 masters receive them after the FP16 handoff
 * (ks3_int8.py:426-429), written straight into a training step's gradient
 * buffer.  Same status behaviour. */
int ksd8_ks3_vjp_reduce_f32(const float* partials, int64_t n_tiles, int64_t charts,
                            const float* raw_scale, const float* raw_shift, float* dcoeff32,
                            float* dscale32, float* dshift32, int* status, void* stream);

/* Pack Rosa symbol bits: bit(stream, t) = x[b*sb + t*st + s*ss] > 0 with
 * stream = b*S + s, into words (streams, ceil(T/64)) uint64, bit t%64 of
 * word t/64.  x_dtype: KSD8_F32 / KSD8_BF16 / KSD8_F16 / KSD8_I8. */
int ksd8_rosa_pack_bits(const void* x, int x_dtype, int64_t batch, int64_t t_len,
                        int64_t streams, int64_t sb, int64_t st, int64_t ss, uint64_t* words,
                        int* status, void* stream);

/* Longest-suffix match per stream (rosa.py:40-98): for each t, the longest
 * L <= max_len with q[t-L+1..t] == k[j-L+1..j], L-1 <= j < t, latest such j;
 * sign = +1 if v[j+1] else -1 (-1 without a match).  out[b*ob + t*ot + s*os]
 * = payload[s] * sign (payload may be NULL = 1) as out_dtype; optional
 * match_len / match_end (streams, T) int32 (0 / -1 without a match). */
int ksd8_rosa_match(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw, int64_t batch,
                    int64_t streams, int64_t t_len, int max_len, const float* payload,
                    void* out, int out_dtype, int64_t ob, int64_t ot, int64_t os,
                    int32_t* match_len, int32_t* match_end, int* status, void* stream);

/* ksd8_rosa_match with scratch (1 + batch * streams int32 of device memory) for
 * the adaptive matcher (algorithm 0): the chunked prefix-table kernel runs
 * every stream, and a stream whose level-12 chain walks exceed a budget (long
 * runs make them O(T) per position) is handed, through the scratch list, to
 * the sorted-key kernel, which rewrites all of its positions.  Same results. */
int ksd8_rosa_match_scratch(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw,
                            int64_t batch, int64_t streams, int64_t t_len, int max_len,
                            const float* payload, void* out, int out_dtype, int64_t ob,
                            int64_t ot, int64_t os, int32_t* match_len, int32_t* match_end,
                            int32_t* scratch, int64_t scratch_len, int* status, void* stream);

/* Matcher kernel behind ksd8_rosa_match (process-wide, identical results):
 * 0 = prefix tables processed 32 positions per warp step, degenerate streams
 * redone by sorted keys (default), 1 = prefix tables one position per step, 2 =
 * window scan, 3 = sorted key windows with a max segment tree (O(log T) per
 * position on any bit statistics; T <= 4096 + max_len - 1, else as 0), 4 =
 * bit-parallel over the k words (64 keys per mask step, O(T / 64 x matched
 * bits) per position).  T >= 8192 takes the bit-parallel kernel (the window
 * scan under 2). */
int ksd8_rosa_set_algorithm(int algo);

/* Counterfactual credits of the hard Rosa core, ksdraft/kernels/rosa_credit_gpu.py:25-48
 * (HardRosaGPU.backward's _chunk_credits; the reference stops at T <= 63):
 * for stream r and every position p, credit_X[r * T + p] = sum over t of
 * (sign'(t) - sign(t)) * grad[r * T + t], sign' the match signs (rosa.py:40-98,
 * cap max_len) with bit X[p] flipped, X = q, k, v; grad (streams, T) fp32 =
 * dL/d sign; bits as ksd8_rosa_pack_bits packs them.  Exact: only the
 * positions a flip can change are re-matched.  Work grows as T^2 per stream
 * (about 64 key comparisons per (flip, later position)); t_len <=
 * KSD8_ROSA_CREDITS_TMAX. */
#define KSD8_ROSA_CREDITS_TMAX 16384
int ksd8_rosa_credits(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw,
                      int64_t streams, int64_t t_len, int max_len, const float* grad,
                      float* credit_q, float* credit_k, float* credit_v, int* status,
                      void* stream);

/* Rosa time-shift mix + per-token GS quantisation of the three projection
 * inputs: x (B, T, d) bf16/f32; mix_q/k/v (d) fp32 = sigmoid(time_mix_*);
 * in_X = prev + (x - prev) * mix_X with (x - prev) rounded to x's dtype.
 * Outputs codes (B*T, d) and scales (B*T, ceil(d/128)) for q, k, v. */
int ksd8_rosa_timemix_quantize(const void* x, int x_dtype, int64_t batch, int64_t t_len,
                               int64_t d, const float* mix_q, const float* mix_k,
                               const float* mix_v, int8_t* q_codes, void* q_scales,
                               int8_t* k_codes, void* k_scales, int8_t* v_codes, void* v_scales,
                               int* status, void* stream);

/* Decoupled-weight-decay Adam over n fp32 parameters with fp16 or fp32
 * gradients (grad_dtype), torch.optim.AdamW semantics (bias-corrected). */
int ksd8_adamw_step(float* param, const void* grad, int grad_dtype, float* exp_avg,
                    float* exp_avg_sq, int64_t n, float lr, float beta1, float beta2, float eps,
                    float weight_decay, int step, int* status, void* stream);

/* The same step with the gradient multiplied by *grad_scale (device memory):
 * the clip coefficient of ksd8_grad_clip_coef, applied without a host round
 * trip (torch.nn.utils.clip_grad_norm_ then AdamW, ksdraft/train/__init__.py:165-166). */
int ksd8_adamw_step_scaled(float* param, const void* grad, int grad_dtype, float* exp_avg,
                           float* exp_avg_sq, int64_t n, float lr, float beta1, float beta2,
                           float eps, float weight_decay, int step, const float* grad_scale,
                           int* status, void* stream);

/* ksd8_adamw_step (grad_scale NULL) or ksd8_adamw_step_scaled over `count`
 * (<= KSD8_ADAMW_MULTI) tensors in one launch; the pointer and size arrays are
 * host memory, all gradients of one dtype.  Same arithmetic per element. */
#define KSD8_ADAMW_MULTI 8
int ksd8_adamw_multi(int count, float* const* params, const void* const* grads, int grad_dtype,
                     float* const* exp_avgs, float* const* exp_avg_sqs, const int64_t* numels,
                     float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                     const float* grad_scale, int* status, void* stream);

/* Global L2 norm of n fp32 gradients and torch's clip coefficient:
 * out[0] = norm, out[1] = min(1, max_norm / (norm + 1e-6))
 * (torch.nn.utils.clip_grad_norm_, ksdraft/train/__init__.py:165).  scratch:
 * 592 floats of device memory; the partial sums are added in a fixed order. */
#define KSD8_GRAD_CLIP_SCRATCH 592
int ksd8_grad_clip_coef(const float* grad, int64_t n, float max_norm, float* scratch,
                        float* out, int* status, void* stream);

/* Parity probe: out[i] = bits of the fp16 tanh the KS3 kernels use for the
 * fp16 value with bits i, i < n <= 0x7C00 (correctly rounded; the reference's
 * CPU torch.tanh on fp16, ksdraft/kernels/ks3_int8.py:366-367, gives the same). */
int ksd8_fp16_tanh_table(int64_t n, uint16_t* out, void* stream);

/* ---- DSpine injection + ln_ffn, transfer-space loss rows ----
 *
 * Row-major (M, d) tensors of dtype KSD8_F32 / KSD8_BF16 / KSD8_F16 (the
 * activation dtype T), d a multiple of 128 and at most 2048, every pointer
 * 16-byte aligned.  fp32 arithmetic inside; gate_bias, ln_w, ln_b are fp32
 * masters, rounded to T first (a T-typed module's parameters). */

/* h2 = T(h + sigmoid(zsum + gate_bias) * inj);  out = T(LayerNorm(h2) * ln_w + ln_b)
 * (biased variance, eps), mean / rstd (M) fp32 saved for the backward.
 * zsum = gate_q(h) + gate_p(p_prev) and inj = inject(p_prev) are the caller's
 * low-rank GEMM outputs (spine.py:66-69). */
int ksd8_dspine_ln_fwd(const void* h, const void* zsum, const void* inj, int dtype, int64_t m,
                       int64_t d, const float* gate_bias, const float* ln_w, const float* ln_b,
                       float eps, void* h2, void* out, float* mean, float* rstd, int* status,
                       void* stream);

/* Backward of ksd8_dspine_ln_fwd given db = dL/d(out) (T) and dres = the
 * gradient reaching h2 directly (fp32, the block's residual):
 *   dh2 = dres + LayerNorm backward of db (fp32),
 *   dinj = T(dh2 g),  dz = T(dh2 inj g (1 - g)),  g = sigmoid(zsum + gate_bias);
 * column sums into partials (n_parts, 3, d) fp32: [0] sum db * xhat (ln_w grad),
 * [1] sum db (ln_b grad), [2] sum dz (gate_bias grad); the caller adds the
 * n_parts rows (each covers ceil(M / n_parts) consecutive tokens). */
int ksd8_dspine_ln_bwd(const void* h2, const float* mean, const float* rstd, const void* db,
                       const float* dres, const void* zsum, const void* inj, int dtype, int64_t m,
                       int64_t d, const float* gate_bias, const float* ln_w, float* dh2, void* dz,
                       void* dinj, float* partials, int64_t n_parts, int* status, void* stream);

/* Transfer-space rows: norm[t] = |p_t|, dot[t] = <p_t, e_t> and
 * term[t] = 1 - dot[t] / max(norm[t], 1e-12), for p (M, d) of dtype T and the
 * normalised next-token embeddings e (M, d) fp32. */
int ksd8_transfer_rows(const void* p, int dtype, const float* e, int64_t m, int64_t d,
                       float* norm, float* dot, float* term, int* status, void* stream);

/* Gradient of coef * sum_t term[t]:  dp = T(coef * dterm/dp + pgrad + first[t / t_len]
 * on the rows t % t_len == 0) and e_grad -= coef * p_t / max(|p_t|, 1e-12).
 * pgrad (M, d) T and first (M / t_len, d) fp32 are optional addends (NULL). */
int ksd8_transfer_bwd(const void* p, int dtype, const float* e, const float* norm,
                      const float* dot, int64_t m, int64_t d, float coef, const void* pgrad,
                      const float* first, int64_t t_len, void* dp, float* e_grad, int* status,
                      void* stream);

/* Training hard path, gradient of the Rosa payload: o = payload * sign (M, S)
 * (the out_proj input, dtype F32 / BF16 / F16), its GS128 codes (M, S) int8,
 * gx = dL/d(dequantised o) (M, S) fp32, sign (M, S) in o's dtype.  The
 * Int8Linear STE input gradient do = gx + the GS128 scale term (elements tied
 * at the group's amax: sign(o) fp16(sum gx * codes) / 127 / n_tied, inside the
 * clamp range) is reduced to partials[p][s] = sum over the rows of chunk p of
 * do * sign (n_parts chunks of ceil(M / n_parts) rows); the caller adds the
 * rows.  streams a multiple of 4, at most 2048 (the last GS128 group is
 * zero-padded when streams % 128 != 0, as the quantiser pads). */
int ksd8_rosa_payload_bwd(const void* o, const int8_t* codes, const float* gx, const void* sign,
                          int dtype, int64_t m, int64_t streams, float* partials,
                          int64_t n_parts, int* status, void* stream);

/* ---- incremental Rosa matching (drafting) ----
 *
 * State of one (context, stream) row, all caller-allocated device memory:
 *   q / k / v bit histories, (contexts * streams, nw) uint64, bit t of row r in
 *   word t / 64 at bit t % 64 (the ksd8_rosa_pack_bits layout), zero beyond the
 *   positions written;
 *   the main run: sw (rows, cap) uint64 sorted key windows, sj (rows, cap)
 *   uint16 their positions, blk (rows, cap / 64) uint16 max(position + 1) per
 *   64 ranks, smp (rows, cap / 64 + cap / 8) uint64 its sample index (the
 *   windows of every 64th rank, then of every 8th rank); cap a multiple of 64.
 * Keys 0 .. n_main - 1 are the matched context (main run = keys
 * max_len - 1 .. n_main - 1; the earlier ones are compared directly), keys
 * n_main .. t - 1 the delta since the last build, also compared directly.
 * Results equal ksd8_rosa_match on the whole sequence when the sequence has at
 * least max_len + 1 positions (the reference's cap min(62, T - 1) is then
 * max_len = 62). */

/* Sort the keys max_len - 1 .. n_keys - 1 of every row of kw into (sw, sj, blk,
 * smp); n_keys <= cap, smem-limited to n_keys - max_len + 1 <= 16384 keys. */
int ksd8_rosa_decode_build(const uint64_t* kw, int64_t n_streams, int64_t nw, int64_t n_keys,
                           int max_len, uint64_t* sw, uint16_t* sj, uint16_t* blk,
                           uint64_t* smp, int64_t cap, int* status, void* stream);

/* The main run of keys max_len - 1 .. n_new - 1 from the run of keys
 * max_len - 1 .. n_old - 1 in (sw_in, sj_in) (a copy: sw / sj are written)
 * and the k bits of the keys appended since: those keys are sorted and merged
 * in; blk and smp are recomputed.  n_new - max(n_old, max_len - 1) <= 8192. */
int ksd8_rosa_decode_merge(const uint64_t* kw, int64_t n_streams, int64_t nw, int64_t n_old,
                           int64_t n_new, int max_len, const uint64_t* sw_in,
                           const uint16_t* sj_in, uint64_t* sw, uint16_t* sj, uint16_t* blk,
                           uint64_t* smp, int64_t cap, int* status, void* stream);

/* Append k_new (1..32) positions t0 .. t0 + k_new - 1 to every row (bits =
 * proj > 0 of the projections (contexts, k_new, streams), dtype F32 / BF16 /
 * F16; positions >= t0 are overwritten, so t0 may also roll back to any
 * length >= n_main; all three proj NULL: the bits are already in the
 * histories) and write, for new position i, payload[s] * sign to
 * out[c * out_cs + i * streams + s] and optionally the match length / latest
 * endpoint to match_len / match_end[row * ml_rs + i] int32.  pos (device
 * int64 [t0, n_main], or NULL): the kernel reads t0 and n_main there instead
 * (a CUDA graph replays the launch at every position); the host arguments must
 * hold the same values when the launch is recorded or made.  Returns
 * KSD8_ERR_UNSUPPORTED when the delta n_main .. t0 + k_new - 2 outgrows the
 * kernel's 34-word window (about 2000 keys): rebuild with n_keys = t0 first. */
int ksd8_rosa_decode_step(const void* proj_q, const void* proj_k, const void* proj_v, int dtype,
                          int64_t contexts, int64_t streams, int64_t k_new, int64_t t0,
                          int64_t n_main, int max_len, uint64_t* qw, uint64_t* kw, uint64_t* vw,
                          int64_t nw, const uint64_t* sw, const uint16_t* sj,
                          const uint16_t* blk, const uint64_t* smp, int64_t cap,
                          const float* payload, void* out, int64_t out_cs, int out_dtype,
                          int32_t* match_len, int32_t* match_end, int64_t ml_rs,
                          const int64_t* pos, int* status, void* stream);

/* Philox4x32-10 uniform stream used by the dither: out[i] = (word(seed, offset+i) >> 8) * 2^-24. */
int ksd8_philox_uniform(uint64_t seed, uint64_t offset, int64_t n, float* out, void* stream);

/* ---- LM head: vocab-parallel cross-entropy and top-k ----
 *
 * The reference head is the tied fp32 nn.Linear(d, V) + F.cross_entropy of
 * ksdraft/model/draft.py:39,51,82 and ksdraft/train/__init__.py:77.  With the
 * vocabulary split into contiguous shards (one per rank) the logits shard
 * (M, V_local) comes from ksd8_w8a8_gemm; these entry points reduce it. */

/* Per row of the shard: out_max = max_c l, out_sum = sum_c exp(l - out_max),
 * out_tgt = l[targets[row] - vstart] when that column is in the shard, else 0.
 * logits (M, V_local) row stride ld, dtype KSD8_F32 / KSD8_BF16 / KSD8_F16;
 * targets (M) int64 global vocab ids; outputs (M) fp32. */
int ksd8_ce_partials(const void* logits, int dtype, int64_t m, int64_t v_local, int64_t ld,
                     const int64_t* targets, int64_t vstart, float* out_max, float* out_sum,
                     float* out_tgt, int* status, void* stream);

/* dlogits[row, c] = (exp(l - gmax[row]) / gsum[row] - [vstart + c == targets[row]]) * scale,
 * the cross-entropy gradient of the shard given the global max and sum of
 * exp over all shards (scale = 1 / total rows for the mean reduction).
 * dlogits fp32 (M, V_local) row stride ldd. */
int ksd8_ce_grad(const void* logits, int dtype, int64_t m, int64_t v_local, int64_t ld,
                 const int64_t* targets, int64_t vstart, const float* gmax, const float* gsum,
                 float scale, float* dlogits, int64_t ldd, int* status, void* stream);

/* ksd8_ce_grad's dlogits quantised straight into the two backward GEMM
 * operands, without writing dlogits: dq (M, Vp) codes along the vocabulary
 * (row stride ldq >= Vp = ceil(V_local/128)*128) with dq_scales (M, Vp/128)
 * fp16, and dqt (V_local, Mp) codes along the tokens (row stride ldqt >= Mp =
 * ceil(M/128)*128) with dqt_scales (V_local, Mp/128) fp16 -- the same codes as
 * ksd8_quantize_rows / ksd8_quantize_cols of the fp32 dlogits; the padded
 * tails are zero codes. */
int ksd8_ce_grad_quant(const void* logits, int dtype, int64_t m, int64_t v_local, int64_t ld,
                       const int64_t* targets, int64_t vstart, const float* gmax,
                       const float* gsum, float scale, int8_t* dq, int64_t ldq, void* dq_scales,
                       int8_t* dqt, int64_t ldqt, void* dqt_scales, int* status, void* stream);

/* Per-row top-k (1 <= k <= 32) of vals (M, C) row stride ld: out_vals (M, k)
 * fp32 descending, out_ids (M, k) int64; ids are offset + column, or idx[row,
 * column] when idx (M, C, same stride) is given (merging gathered shard
 * candidates).  Ties: the smaller id first. */
int ksd8_topk_rows(const void* vals, int dtype, const int64_t* idx, int64_t m, int64_t c,
                   int64_t ld, int k, int64_t offset, float* out_vals, int64_t* out_ids,
                   int* status, void* stream);

/* ---- allocation-free variant (no counterpart in the reference) ----
 *
 * ksd8_ks3_vjp_static: ksd8_ks3_vjp followed by ksd8_ks3_vjp_reduce, with the
 * (n_tiles, 8, charts) fp32 partials held in a file-scope static device array
 * of KSD8_VJP_STATIC_MAX_PARTIALS floats (8 MiB) instead of caller scratch.
 * The reference has no such entry point: its backward (ks3_int8.py:354-395)
 * lets torch allocate the intermediate.  This one allocates nothing (no
 * cudaMalloc / cudaFree, no library allocator) and writes the same outputs,
 * bit for bit, as the two-call path.
 * Who needs it: code that drives the backward through this C ABI from
 * another runtime -- an FFI binding or plugin host that is handed its device
 * buffers by an owner which reserved all device memory up front -- has no
 * allocator to get the partials buffer from, and calling cudaMalloc in the
 * middle of a training step would also stall the device for every stream.
 *   - Limit: ceil(m / 128) * 8 * charts <= KSD8_VJP_STATIC_MAX_PARTIALS, e.g.
 *     m = 4096 tokens with up to 8192 charts; larger requests return
 *     KSD8_ERR_SCRATCH_LIMIT before anything launches.
 *   - Set-up: the first call on each device (with that device current) looks
 *     up the array's device address once with cudaGetSymbolAddress and caches
 *     it; make that first call before any stream capture on the device.
 *     The cache is never refreshed, so a device reset (cudaDeviceReset) after
 *     the first call is not supported.  Devices 0..31 only (as ksd8_ks3_vjp).
 *   - Nothing in the scratch needs clearing: the VJP writes every partial the
 *     reduction then reads.
 *   - Calls that overlap on one device (other streams, other host threads)
 *     share the one array and race; serialise them.
 * Arguments are those of ksd8_ks3_vjp (minus partials) and of
 * ksd8_ks3_vjp_reduce (minus partials, n_tiles); status may be NULL. */
#define KSD8_VJP_STATIC_MAX_PARTIALS (1 << 21)
#define KSD8_ERR_SCRATCH_LIMIT 9 /* request exceeds a static scratch array */
int ksd8_ks3_vjp_static(const void* value, const void* coords, int64_t m, int64_t charts,
                        const int8_t* spine_codes, const void* spine_scale,
                        const int8_t* warp_scale_codes, const void* warp_scale_scales,
                        const int8_t* warp_shift_codes, const void* warp_shift_scales,
                        int8_t* dc_codes, void* dc_scales, int8_t* dct_codes, void* dct_scales,
                        const float* raw_scale, const float* raw_shift, void* dcoeff16,
                        void* dscale16, void* dshift16, int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KSD8_H_ */
