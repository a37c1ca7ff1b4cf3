// extern "C" boundary of libksd8: argument validation on the host, then the
// launches of quant.cu / gemm_sm100.cu / ks3.cu / rosa.cu on the caller's stream.
// Shape, dtype and alignment errors return a status before anything launches.
#include <atomic>
#include <cstdio>

#include "common.cuh"

// launchers defined in the kernel translation units
int ksd8_quantize_rows_launch(const void*, int, int64_t, int64_t, int64_t, int, int, float,
                              uint64_t, uint64_t, int8_t*, int64_t, void*, int*, cudaStream_t);
int ksd8_quantize_cols_launch(const void*, int, const void*, int, int64_t, int64_t, int64_t, int,
                              int8_t*, int64_t, void*, int*, cudaStream_t);
int ksd8_philox_launch(uint64_t, uint64_t, int64_t, float*, cudaStream_t);
int ksd8_fp16_tanh_table_launch(int64_t, uint16_t*, cudaStream_t);
int ksd8_rosa_algorithm(int);
int ksd8_gemm_launch(const int8_t*, const void*, const int8_t*, const void*, int64_t, int64_t,
                     int64_t, void*, int, int64_t, const float*, int, int*, cudaStream_t, bool);
int ksd8_ks3_pack_launch(const float*, const float*, const float*, int64_t, int8_t*, void*,
                         int8_t*, void*, int8_t*, void*, cudaStream_t);
int ksd8_ks3_spine_table_launch(int64_t, const int8_t*, const void*, const int8_t*, const void*,
                                const int8_t*, const void*, const int8_t*, void*, cudaStream_t);
int ksd8_ks3_spine_quant_launch(const void*, int64_t, int64_t, const int8_t*, const void*,
                                const int8_t*, const void*, const int8_t*, const void*,
                                const int8_t*, int, const void*, int8_t*, void*, cudaStream_t);
int ksd8_ks3_vjp_launch(const void*, const void*, int64_t, int64_t, const int8_t*, const void*,
                        const int8_t*, const void*, const int8_t*, const void*, int8_t*, void*,
                        int8_t*, void*, float*, int*, cudaStream_t);
int ksd8_ks3_vjp_reduce_launch(const float*, int64_t, int64_t, const float*, const float*, void*,
                               void*, void*, int*, cudaStream_t, float*, float*, float*);
int ksd8_rosa_pack_bits_launch(const void*, int, int64_t, int64_t, int64_t, int64_t, int64_t,
                               int64_t, uint64_t*, cudaStream_t);
int ksd8_rosa_credits_launch(const uint64_t*, const uint64_t*, const uint64_t*, int64_t, int64_t,
                             int, const float*, float*, float*, float*, cudaStream_t);
int ksd8_rosa_match_launch(const uint64_t*, const uint64_t*, const uint64_t*, int64_t, int64_t,
                           int64_t, int, const float*, void*, int, int64_t, int64_t, int64_t,
                           int32_t*, int32_t*, cudaStream_t, int32_t*);
int ksd8_rosa_timemix_launch(const void*, int, int64_t, int64_t, int64_t, const float*,
                             const float*, const float*, int8_t*, void*, int8_t*, void*, int8_t*,
                             void*, cudaStream_t);
int ksd8_ce_partials_launch(const void*, int, int64_t, int64_t, int64_t, const int64_t*, int64_t,
                            float*, float*, float*, cudaStream_t);
int ksd8_ce_grad_launch(const void*, int, int64_t, int64_t, int64_t, const int64_t*, int64_t,
                        const float*, const float*, float, float*, int64_t, cudaStream_t);
int ksd8_topk_rows_launch(const void*, int, const int64_t*, int64_t, int64_t, int64_t, int, int64_t,
                          float*, int64_t*, cudaStream_t);
int ksd8_ce_grad_quant_launch(const void*, int, int64_t, int64_t, int64_t, const int64_t*, int64_t,
                              const float*, const float*, float, int8_t*, int64_t, void*, int8_t*,
                              int64_t, void*, cudaStream_t);
int ksd8_adamw_launch(float*, const void*, int, float*, float*, int64_t, float, float, float,
                      float, float, int, cudaStream_t, const float*);
int ksd8_grad_clip_launch(const float*, int64_t, float, float*, float*, cudaStream_t);
int ksd8_dspine_ln_fwd_launch(const void*, const void*, const void*, int, int64_t, int64_t,
                              const float*, const float*, const float*, float, void*, void*,
                              float*, float*, cudaStream_t);
int ksd8_dspine_ln_bwd_launch(const void*, const float*, const float*, const void*, const float*,
                              const void*, const void*, int, int64_t, int64_t, const float*,
                              const float*, float*, void*, void*, float*, int64_t, cudaStream_t);
int ksd8_transfer_rows_launch(const void*, int, const float*, int64_t, int64_t, float*, float*,
                              float*, cudaStream_t);
int ksd8_rosa_decode_build_launch(const uint64_t*, int64_t, int64_t, int64_t, int, uint64_t*,
                                  uint16_t*, uint16_t*, uint64_t*, int64_t, cudaStream_t);
int ksd8_rosa_decode_step_launch(const void* const*, int, int64_t, int64_t, int64_t, int64_t,
                                 int64_t, int, uint64_t* const*, int64_t, const uint64_t*,
                                 const uint16_t*, const uint16_t*, const uint64_t*, int64_t,
                                 const float*, void*,
                                 int64_t, int, int32_t*, int32_t*, int64_t, const int64_t*,
                                 cudaStream_t);
int ksd8_rosa_decode_limits(int64_t*, int64_t*, int64_t*);
int ksd8_rosa_payload_bwd_launch(const void*, const int8_t*, const float*, const void*, int,
                                 int64_t, int64_t, float*, int64_t, cudaStream_t);
int ksd8_rosa_decode_merge_launch(const uint64_t*, int64_t, int64_t, int64_t, int64_t, int,
                                  const uint64_t*, const uint16_t*, uint64_t*, uint16_t*,
                                  uint16_t*, uint64_t*, int64_t, cudaStream_t);
int ksd8_transfer_bwd_launch(const void*, int, const float*, const float*, const float*, int64_t,
                             int64_t, float, const void*, const float*, int64_t, void*, float*,
                             cudaStream_t);
int ksd8_adamw_multi_launch(int, float* const*, const void* const*, int, float* const*,
                            float* const*, const int64_t*, float, float, float, float, float,
                            int, const float*, cudaStream_t);

static thread_local int g_last_cuda_error = 0;

static int finish(int rc) {
  if (rc != KSD8_OK) return rc;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return KSD8_ERR_LAUNCH;
  }
  return KSD8_OK;
}

static inline bool valid_float_dtype(int d) {
  return d == KSD8_F32 || d == KSD8_F16 || d == KSD8_BF16;
}

static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

int ksd8_version(void) { return 1; }

const char* ksd8_status_string(int status) {
  switch (status) {
    case KSD8_OK: return "ok";
    case KSD8_ERR_SHAPE: return "shape mismatch";
    case KSD8_ERR_ALIGN: return "misaligned pointer or stride";
    case KSD8_ERR_DTYPE: return "unsupported dtype";
    case KSD8_ERR_LAUNCH: return "CUDA launch failure";
    case KSD8_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case KSD8_ERR_UNSUPPORTED: return "unsupported configuration";
    case KSD8_ERR_ARG: return "invalid argument";
    case KSD8_ERR_NONFINITE: return "non-finite fp16 output";
    case KSD8_ERR_SCRATCH_LIMIT: return "request exceeds the static scratch capacity";
    default: return "unknown status";
  }
}

int ksd8_last_cuda_error(void) { return g_last_cuda_error; }

static std::atomic<int> g_sm_reserve{0};

int ksd8_set_sm_reserve(int n) {
  if (n < 0 || n > 1024) return KSD8_ERR_ARG;
  g_sm_reserve.store(n);
  return KSD8_OK;
}

int ksd8_get_sm_reserve(void) { return g_sm_reserve.load(); }

int ksd8_sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}

int ksd8_quantize_rows(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t ldx,
                       int group, int flags, float dither, uint64_t seed, uint64_t offset,
                       int8_t* codes, int64_t ldc, void* scales, int* status, void* stream) {
  if (!valid_float_dtype(x_dtype)) return KSD8_ERR_DTYPE;
  if (group != 128) return KSD8_ERR_UNSUPPORTED;
  if (rows < 0 || k < 0 || ldx < k || ldc < k) return KSD8_ERR_SHAPE;
  if ((rows > 0 && k > 0) && (!x || !codes || !scales)) return KSD8_ERR_ARG;
  if ((flags & KSD8_Q_DITHER) && !(dither >= 0.f)) return KSD8_ERR_ARG;
  return finish(ksd8_quantize_rows_launch(x, x_dtype, rows, k, ldx, group, flags, dither, seed,
                                          offset, codes, ldc, scales, status, S(stream)));
}

int ksd8_quantize_cols(const void* x, int x_dtype, const void* x_scales, int x_group,
                       int64_t rows, int64_t cols, int64_t ldx, int group, int flags,
                       int8_t* codes_t, int64_t ldct, void* scales_t, int* status, void* stream) {
  if (!(valid_float_dtype(x_dtype) || x_dtype == KSD8_I8)) return KSD8_ERR_DTYPE;
  if (group != 128) return KSD8_ERR_UNSUPPORTED;
  if (x_dtype == KSD8_I8 && (!x_scales || x_group <= 0)) return KSD8_ERR_ARG;
  if (x_dtype == KSD8_I8 && (x_group % 128) != 0) return KSD8_ERR_UNSUPPORTED;
  if (rows < 0 || cols < 0 || ldx < cols || ldct < rows) return KSD8_ERR_SHAPE;
  if ((rows > 0 && cols > 0) && (!x || !codes_t || !scales_t)) return KSD8_ERR_ARG;
  return finish(ksd8_quantize_cols_launch(x, x_dtype, x_scales, x_group, rows, cols, ldx, flags,
                                          codes_t, ldct, scales_t, status, S(stream)));
}

int ksd8_w8a8_gemm(const int8_t* a, const void* a_scales, const int8_t* w, const void* w_scales,
                   int64_t m, int64_t n, int64_t k, int group, void* out, int out_dtype,
                   int64_t ldo, const float* bias, int epi_flags, int* status, void* stream) {
  if (group != 128) return KSD8_ERR_UNSUPPORTED;
  if (!valid_float_dtype(out_dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || n < 0 || k < 0 || (k % 128) != 0 || ldo < n) return KSD8_ERR_SHAPE;
  if (m > INT32_MAX || n > INT32_MAX) return KSD8_ERR_SHAPE;
  if (m == 0 || n == 0) return KSD8_OK;
  if (!a || !w || !a_scales || !w_scales || !out) return KSD8_ERR_ARG;
  if ((epi_flags & KSD8_EPI_BIAS) && !bias) return KSD8_ERR_ARG;
  if ((epi_flags & KSD8_EPI_IF_STATUS) && !status) return KSD8_ERR_ARG;
  if ((epi_flags & KSD8_EPI_ROUND_F16) && out_dtype != KSD8_F32) return KSD8_ERR_ARG;
  // TMA: 16-byte aligned base addresses (row pitch k is a multiple of 128).
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return KSD8_ERR_ALIGN;
  if (k == 0) return KSD8_ERR_SHAPE;
  return finish(ksd8_gemm_launch(a, a_scales, w, w_scales, m, n, k, out, out_dtype, ldo, bias,
                                 epi_flags, status, S(stream), false));
}

int ksd8_w8a8_group_partials(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                             int32_t* out, int* status, void* stream) {
  if (m <= 0 || n <= 0 || k <= 0 || (k % 128) != 0) return KSD8_ERR_SHAPE;
  if (!a || !w || !out) return KSD8_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return KSD8_ERR_ALIGN;
  // The scale operands are unused in this mode but the loader reads them:
  // point them at the codes (any readable memory of sufficient size is fine).
  return finish(ksd8_gemm_launch(a, nullptr, w, nullptr, m, n, k, out, KSD8_F32, n, nullptr, 0,
                                 status, S(stream), true));
}

int ksd8_ks3_pack(const float* coefficients, const float* raw_scale, const float* raw_shift,
                  int64_t charts, int8_t* spine_codes, void* spine_scale,
                  int8_t* warp_scale_codes, void* warp_scale_scales, int8_t* warp_shift_codes,
                  void* warp_shift_scales, int* status, void* stream) {
  (void)status;
  if (charts < 0) return KSD8_ERR_SHAPE;
  if (charts > 0 && (!coefficients || !raw_scale || !raw_shift || !spine_codes || !spine_scale ||
                     !warp_scale_codes || !warp_scale_scales || !warp_shift_codes ||
                     !warp_shift_scales))
    return KSD8_ERR_ARG;
  return finish(ksd8_ks3_pack_launch(coefficients, raw_scale, raw_shift, charts, spine_codes,
                                     spine_scale, warp_scale_codes, warp_scale_scales,
                                     warp_shift_codes, warp_shift_scales, S(stream)));
}

int ksd8_ks3_spine_table(int64_t charts, const int8_t* spine_codes, const void* spine_scale,
                         const int8_t* warp_scale_codes, const void* warp_scale_scales,
                         const int8_t* warp_shift_codes, const void* warp_shift_scales,
                         const int8_t* lut, void* table, int* status, void* stream) {
  (void)status;
  if (charts < 0) return KSD8_ERR_SHAPE;
  if (charts > 0 && (!spine_codes || !spine_scale || !warp_scale_scales || !warp_shift_scales ||
                     !lut || !table))
    return KSD8_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(table) & 15) return KSD8_ERR_ALIGN;
  return finish(ksd8_ks3_spine_table_launch(charts, spine_codes, spine_scale, warp_scale_codes,
                                            warp_scale_scales, warp_shift_codes,
                                            warp_shift_scales, lut, table, S(stream)));
}

int ksd8_ks3_spine_quant(const void* coords, int64_t m, int64_t charts,
                         const int8_t* spine_codes, const void* spine_scale,
                         const int8_t* warp_scale_codes, const void* warp_scale_scales,
                         const int8_t* warp_shift_codes, const void* warp_shift_scales,
                         const int8_t* lut, int nonlinear, const void* table, int8_t* h_codes,
                         void* h_scales, int* status, void* stream) {
  (void)status;
  if (nonlinear < KSD8_NL_FP32 || nonlinear > KSD8_NL_INT8) return KSD8_ERR_ARG;
  if (m < 0 || charts < 0) return KSD8_ERR_SHAPE;
  if (m > 0 && charts > 0 && !table &&
      (!coords || !spine_codes || !spine_scale || !warp_scale_scales || !warp_shift_scales ||
       !lut || !h_codes || !h_scales))
    return KSD8_ERR_ARG;
  if (m > 0 && charts > 0 && (!coords || !h_codes || !h_scales)) return KSD8_ERR_ARG;
  if (table && (reinterpret_cast<uintptr_t>(table) & 15)) return KSD8_ERR_ALIGN;
  return finish(ksd8_ks3_spine_quant_launch(coords, m, charts, spine_codes, spine_scale,
                                            warp_scale_codes, warp_scale_scales, warp_shift_codes,
                                            warp_shift_scales, lut, nonlinear, table, h_codes,
                                            h_scales, S(stream)));
}

int ksd8_ks3_vjp(const void* value, const void* coords, int64_t m, int64_t charts,
                 const int8_t* spine_codes, const void* spine_scale,
                 const int8_t* warp_scale_codes, const void* warp_scale_scales,
                 const int8_t* warp_shift_codes, const void* warp_shift_scales,
                 int8_t* dc_codes, void* dc_scales, int8_t* dct_codes, void* dct_scales,
                 float* partials, int* status, void* stream) {
  if (m < 0 || charts <= 0 || (charts % 128) != 0) return KSD8_ERR_SHAPE;
  if (m > 0 && (!value || !coords || !spine_codes || !spine_scale || !warp_scale_codes ||
                !warp_scale_scales || !warp_shift_codes || !warp_shift_scales || !dc_codes ||
                !dc_scales || !dct_codes || !dct_scales || !partials))
    return KSD8_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(value) & 15) || (reinterpret_cast<uintptr_t>(coords) & 15) ||
      (reinterpret_cast<uintptr_t>(dc_codes) & 3))
    return KSD8_ERR_ALIGN;
  return finish(ksd8_ks3_vjp_launch(value, coords, m, charts, spine_codes, spine_scale,
                                    warp_scale_codes, warp_scale_scales, warp_shift_codes,
                                    warp_shift_scales, dc_codes, dc_scales, dct_codes, dct_scales,
                                    partials, status, S(stream)));
}

int ksd8_ks3_vjp_reduce(const float* partials, int64_t n_tiles, int64_t charts,
                        const float* raw_scale, const float* raw_shift, void* dcoeff16,
                        void* dscale16, void* dshift16, int* status, void* stream) {
  if (n_tiles < 0 || charts < 0) return KSD8_ERR_SHAPE;
  if (charts > 0 && (!partials || !raw_scale || !raw_shift || !dcoeff16 || !dscale16 ||
                     !dshift16))
    return KSD8_ERR_ARG;
  return finish(ksd8_ks3_vjp_reduce_launch(partials, n_tiles, charts, raw_scale, raw_shift,
                                           dcoeff16, dscale16, dshift16, status, S(stream),
                                           nullptr, nullptr, nullptr));
}

int ksd8_ks3_vjp_reduce_f32(const float* partials, int64_t n_tiles, int64_t charts,
                            const float* raw_scale, const float* raw_shift, float* dcoeff32,
                            float* dscale32, float* dshift32, int* status, void* stream) {
  if (n_tiles < 0 || charts < 0) return KSD8_ERR_SHAPE;
  if (charts > 0 && (!partials || !raw_scale || !raw_shift || !dcoeff32 || !dscale32 ||
                     !dshift32))
    return KSD8_ERR_ARG;
  return finish(ksd8_ks3_vjp_reduce_launch(partials, n_tiles, charts, raw_scale, raw_shift,
                                           nullptr, nullptr, nullptr, status, S(stream),
                                           dcoeff32, dscale32, dshift32));
}

int ksd8_rosa_pack_bits(const void* x, int x_dtype, int64_t batch, int64_t t_len,
                        int64_t streams, int64_t sb, int64_t st, int64_t ss, uint64_t* words,
                        int* status, void* stream) {
  (void)status;
  if (!(valid_float_dtype(x_dtype) || x_dtype == KSD8_I8)) return KSD8_ERR_DTYPE;
  if (batch < 0 || t_len < 0 || streams < 0) return KSD8_ERR_SHAPE;
  if (batch * streams * t_len > 0 && (!x || !words)) return KSD8_ERR_ARG;
  return finish(
      ksd8_rosa_pack_bits_launch(x, x_dtype, batch, t_len, streams, sb, st, ss, words, S(stream)));
}

int ksd8_rosa_match(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw, int64_t batch,
                    int64_t streams, int64_t t_len, int max_len, const float* payload,
                    void* out, int out_dtype, int64_t ob, int64_t ot, int64_t os,
                    int32_t* match_len, int32_t* match_end, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(out_dtype)) return KSD8_ERR_DTYPE;
  if (batch < 0 || streams < 0 || t_len < 0) return KSD8_ERR_SHAPE;
  if (max_len < 0 || max_len > 64) return KSD8_ERR_ARG;
  if (t_len > 25600) return KSD8_ERR_UNSUPPORTED;  // key windows must fit in shared memory
  if (batch * streams * t_len > 0 && (!qw || !kw || !vw || !out)) return KSD8_ERR_ARG;
  return finish(ksd8_rosa_match_launch(qw, kw, vw, batch, streams, t_len, max_len, payload, out,
                                       out_dtype, ob, ot, os, match_len, match_end, S(stream),
                                       nullptr));
}

int ksd8_rosa_match_scratch(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw,
                            int64_t batch, int64_t streams, int64_t t_len, int max_len,
                            const float* payload, void* out, int out_dtype, int64_t ob,
                            int64_t ot, int64_t os, int32_t* match_len, int32_t* match_end,
                            int32_t* scratch, int64_t scratch_len, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(out_dtype)) return KSD8_ERR_DTYPE;
  if (batch < 0 || streams < 0 || t_len < 0) return KSD8_ERR_SHAPE;
  if (max_len < 0 || max_len > 64) return KSD8_ERR_ARG;
  if (t_len > 25600) return KSD8_ERR_UNSUPPORTED;
  if (batch * streams * t_len > 0 && (!qw || !kw || !vw || !out)) return KSD8_ERR_ARG;
  if (!scratch || scratch_len < 1 + batch * streams) return KSD8_ERR_SHAPE;
  return finish(ksd8_rosa_match_launch(qw, kw, vw, batch, streams, t_len, max_len, payload, out,
                                       out_dtype, ob, ot, os, match_len, match_end, S(stream),
                                       scratch));
}

int ksd8_rosa_credits(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw,
                      int64_t streams, int64_t t_len, int max_len, const float* grad,
                      float* credit_q, float* credit_k, float* credit_v, int* status,
                      void* stream) {
  (void)status;
  if (streams < 0 || t_len < 0) return KSD8_ERR_SHAPE;
  if (max_len < 0 || max_len > 64) return KSD8_ERR_ARG;
  if (t_len > KSD8_ROSA_CREDITS_TMAX) return KSD8_ERR_UNSUPPORTED;
  if (streams * t_len > 0 && (!qw || !kw || !vw || !grad || !credit_q || !credit_k || !credit_v))
    return KSD8_ERR_ARG;
  return finish(ksd8_rosa_credits_launch(qw, kw, vw, streams, t_len, max_len, grad, credit_q,
                                         credit_k, credit_v, S(stream)));
}

int ksd8_rosa_timemix_quantize(const void* x, int x_dtype, int64_t batch, int64_t t_len,
                               int64_t d, const float* mix_q, const float* mix_k,
                               const float* mix_v, int8_t* q_codes, void* q_scales,
                               int8_t* k_codes, void* k_scales, int8_t* v_codes, void* v_scales,
                               int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(x_dtype)) return KSD8_ERR_DTYPE;
  if (batch < 0 || t_len < 0 || d < 0) return KSD8_ERR_SHAPE;
  if (batch * t_len * d > 0 && (!x || !mix_q || !mix_k || !mix_v || !q_codes || !q_scales ||
                                !k_codes || !k_scales || !v_codes || !v_scales))
    return KSD8_ERR_ARG;
  return finish(ksd8_rosa_timemix_launch(x, x_dtype, batch, t_len, d, mix_q, mix_k, mix_v,
                                         q_codes, q_scales, k_codes, k_scales, v_codes, v_scales,
                                         S(stream)));
}

int ksd8_adamw_step(float* param, const void* grad, int grad_dtype, float* exp_avg,
                    float* exp_avg_sq, int64_t n, float lr, float beta1, float beta2, float eps,
                    float weight_decay, int step, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(grad_dtype)) return KSD8_ERR_DTYPE;
  if (n < 0) return KSD8_ERR_SHAPE;
  if (step < 1) return KSD8_ERR_ARG;
  if (n > 0 && (!param || !grad || !exp_avg || !exp_avg_sq)) return KSD8_ERR_ARG;
  return finish(ksd8_adamw_launch(param, grad, grad_dtype, exp_avg, exp_avg_sq, n, lr, beta1,
                                  beta2, eps, weight_decay, step, S(stream), nullptr));
}

int ksd8_adamw_step_scaled(float* param, const void* grad, int grad_dtype, float* exp_avg,
                           float* exp_avg_sq, int64_t n, float lr, float beta1, float beta2,
                           float eps, float weight_decay, int step, const float* grad_scale,
                           int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(grad_dtype)) return KSD8_ERR_DTYPE;
  if (n < 0) return KSD8_ERR_SHAPE;
  if (step < 1) return KSD8_ERR_ARG;
  if (n > 0 && (!param || !grad || !exp_avg || !exp_avg_sq || !grad_scale)) return KSD8_ERR_ARG;
  return finish(ksd8_adamw_launch(param, grad, grad_dtype, exp_avg, exp_avg_sq, n, lr, beta1,
                                  beta2, eps, weight_decay, step, S(stream), grad_scale));
}

int ksd8_adamw_multi(int count, float* const* params, const void* const* grads, int grad_dtype,
                     float* const* exp_avgs, float* const* exp_avg_sqs, const int64_t* numels,
                     float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                     const float* grad_scale, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(grad_dtype)) return KSD8_ERR_DTYPE;
  if (count < 0 || count > KSD8_ADAMW_MULTI) return KSD8_ERR_UNSUPPORTED;
  if (step < 1) return KSD8_ERR_ARG;
  if (count > 0 && (!params || !grads || !exp_avgs || !exp_avg_sqs || !numels))
    return KSD8_ERR_ARG;
  for (int k = 0; k < count; ++k) {
    if (numels[k] < 0) return KSD8_ERR_SHAPE;
    if (numels[k] > 0 && (!params[k] || !grads[k] || !exp_avgs[k] || !exp_avg_sqs[k]))
      return KSD8_ERR_ARG;
  }
  return finish(ksd8_adamw_multi_launch(count, params, grads, grad_dtype, exp_avgs, exp_avg_sqs,
                                        numels, lr, beta1, beta2, eps, weight_decay, step,
                                        grad_scale, S(stream)));
}

int ksd8_grad_clip_coef(const float* grad, int64_t n, float max_norm, float* scratch,
                        float* out, int* status, void* stream) {
  (void)status;
  if (n < 0) return KSD8_ERR_SHAPE;
  if (!(max_norm > 0.f)) return KSD8_ERR_ARG;
  if (!scratch || !out || (n > 0 && !grad)) return KSD8_ERR_ARG;
  return finish(ksd8_grad_clip_launch(grad, n, max_norm, scratch, out, S(stream)));
}

int ksd8_ce_partials(const void* logits, int dtype, int64_t m, int64_t v_local, int64_t ld,
                     const int64_t* targets, int64_t vstart, float* out_max, float* out_sum,
                     float* out_tgt, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || v_local <= 0 || ld < v_local || vstart < 0) return KSD8_ERR_SHAPE;
  if (m > 0 && (!logits || !targets || !out_max || !out_sum || !out_tgt)) return KSD8_ERR_ARG;
  if (m > INT32_MAX) return KSD8_ERR_SHAPE;
  return finish(ksd8_ce_partials_launch(logits, dtype, m, v_local, ld, targets, vstart, out_max,
                                        out_sum, out_tgt, S(stream)));
}

int ksd8_ce_grad(const void* logits, int dtype, int64_t m, int64_t v_local, int64_t ld,
                 const int64_t* targets, int64_t vstart, const float* gmax, const float* gsum,
                 float scale, float* dlogits, int64_t ldd, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || v_local <= 0 || ld < v_local || ldd < v_local || vstart < 0) return KSD8_ERR_SHAPE;
  if (m > 65535) return KSD8_ERR_UNSUPPORTED;  // rows map to grid.y
  if (m > 0 && (!logits || !targets || !gmax || !gsum || !dlogits)) return KSD8_ERR_ARG;
  return finish(ksd8_ce_grad_launch(logits, dtype, m, v_local, ld, targets, vstart, gmax, gsum,
                                    scale, dlogits, ldd, S(stream)));
}

int ksd8_ce_grad_quant(const void* logits, int dtype, int64_t m, int64_t v_local, int64_t ld,
                       const int64_t* targets, int64_t vstart, const float* gmax,
                       const float* gsum, float scale, int8_t* dq, int64_t ldq, void* dq_scales,
                       int8_t* dqt, int64_t ldqt, void* dqt_scales, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  const int64_t vp = (v_local + 127) / 128 * 128, mp = (m + 127) / 128 * 128;
  if (m < 0 || v_local <= 0 || ld < v_local || vstart < 0 || ldq < vp || ldqt < mp)
    return KSD8_ERR_SHAPE;
  if (m > 65535 * 128 || v_local > 2147483647LL * 128) return KSD8_ERR_UNSUPPORTED;  // grid
  if (m > 0 && (!logits || !targets || !gmax || !gsum || !dq || !dq_scales || !dqt ||
                !dqt_scales))
    return KSD8_ERR_ARG;
  return finish(ksd8_ce_grad_quant_launch(logits, dtype, m, v_local, ld, targets, vstart, gmax,
                                          gsum, scale, dq, ldq, dq_scales, dqt, ldqt, dqt_scales,
                                          S(stream)));
}

int ksd8_topk_rows(const void* vals, int dtype, const int64_t* idx, int64_t m, int64_t c,
                   int64_t ld, int k, int64_t offset, float* out_vals, int64_t* out_ids,
                   int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (k < 1 || k > 32) return KSD8_ERR_ARG;
  if (m < 0 || c < k || ld < c) return KSD8_ERR_SHAPE;
  if (m > INT32_MAX) return KSD8_ERR_SHAPE;
  if (m > 0 && (!vals || !out_vals || !out_ids)) return KSD8_ERR_ARG;
  return finish(ksd8_topk_rows_launch(vals, dtype, idx, m, c, ld, k, offset, out_vals, out_ids,
                                      S(stream)));
}

int ksd8_rosa_set_algorithm(int algo) {
  if (algo < 0 || algo > 4) return KSD8_ERR_ARG;
  ksd8_rosa_algorithm(algo);
  return KSD8_OK;
}

int ksd8_fp16_tanh_table(int64_t n, uint16_t* out, void* stream) {
  if (n < 0 || n > 0x7C00) return KSD8_ERR_SHAPE;
  if (n > 0 && !out) return KSD8_ERR_ARG;
  return finish(ksd8_fp16_tanh_table_launch(n, out, S(stream)));
}

int ksd8_philox_uniform(uint64_t seed, uint64_t offset, int64_t n, float* out, void* stream) {
  if (n < 0) return KSD8_ERR_SHAPE;
  if (n > 0 && !out) return KSD8_ERR_ARG;
  return finish(ksd8_philox_launch(seed, offset, n, out, S(stream)));
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free VJP
//
// ksd8_ks3_vjp_static: the VJP and its reduction with the partials in a
// file-scope static device array (8 MiB, resident in every device context
// that loads this library), for callers that cannot allocate: a binding or
// plugin host given its device buffers by an owner that reserved the memory
// up front has no allocator of its own, and a cudaMalloc mid-step would stall
// the device.  Its device address is looked up once per device
// with cudaGetSymbolAddress, with that device current, and cached.  The VJP
// writes every (tile, k, chart) partial that the reduction reads, so nothing
// is cleared.  Calls that overlap on one device share the array and race.

#include <mutex>

static __device__ __align__(256) float g_vjp_scratch[KSD8_VJP_STATIC_MAX_PARTIALS];

namespace {
constexpr int kMaxDevices = 32;  // the same device limit as the VJP launcher's per-device state
std::mutex g_vjp_scratch_mu;
float* g_vjp_scratch_ptr[kMaxDevices] = {};

// Device address of g_vjp_scratch on the current device (set-up on first use).
int vjp_scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    g_last_cuda_error = (int)e;
    return KSD8_ERR_LAUNCH;
  }
  if (dev < 0 || dev >= kMaxDevices) return KSD8_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_vjp_scratch_mu);
  if (!g_vjp_scratch_ptr[dev]) {
    float* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_vjp_scratch);
    if (e != cudaSuccess || !ptr) {
      g_last_cuda_error = (int)e;
      return KSD8_ERR_LAUNCH;
    }
    g_vjp_scratch_ptr[dev] = ptr;
  }
  *out = g_vjp_scratch_ptr[dev];
  return KSD8_OK;
}
}  // namespace

extern "C" int ksd8_ks3_vjp_static(const void* value, const void* coords, int64_t m,
                                   int64_t charts, const int8_t* spine_codes,
                                   const void* spine_scale, const int8_t* warp_scale_codes,
                                   const void* warp_scale_scales, const int8_t* warp_shift_codes,
                                   const void* warp_shift_scales, int8_t* dc_codes,
                                   void* dc_scales, int8_t* dct_codes, void* dct_scales,
                                   const float* raw_scale, const float* raw_shift,
                                   void* dcoeff16, void* dscale16, void* dshift16, int* status,
                                   void* stream) {
  if (m < 0 || charts <= 0 || (charts % 128) != 0) return KSD8_ERR_SHAPE;
  const int64_t n_tiles = (m + 127) / 128;
  const int64_t per_tile = 8 * charts;
  if (per_tile > KSD8_VJP_STATIC_MAX_PARTIALS ||
      n_tiles > KSD8_VJP_STATIC_MAX_PARTIALS / per_tile)
    return KSD8_ERR_SCRATCH_LIMIT;
  if (!raw_scale || !raw_shift || !dcoeff16 || !dscale16 || !dshift16) return KSD8_ERR_ARG;
  if (m > 0 && (!value || !coords || !spine_codes || !spine_scale || !warp_scale_codes ||
                !warp_scale_scales || !warp_shift_codes || !warp_shift_scales || !dc_codes ||
                !dc_scales || !dct_codes || !dct_scales))
    return KSD8_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(value) & 15) || (reinterpret_cast<uintptr_t>(coords) & 15) ||
      (reinterpret_cast<uintptr_t>(dc_codes) & 3))
    return KSD8_ERR_ALIGN;
  float* partials = nullptr;
  int rc = vjp_scratch_for_current_device(&partials);
  if (rc != KSD8_OK) return rc;
  rc = finish(ksd8_ks3_vjp_launch(value, coords, m, charts, spine_codes, spine_scale,
                                  warp_scale_codes, warp_scale_scales, warp_shift_codes,
                                  warp_shift_scales, dc_codes, dc_scales, dct_codes, dct_scales,
                                  partials, status, S(stream)));
  if (rc != KSD8_OK) return rc;
  return finish(ksd8_ks3_vjp_reduce_launch(partials, n_tiles, charts, raw_scale, raw_shift,
                                           dcoeff16, dscale16, dshift16, status, S(stream),
                                           nullptr, nullptr, nullptr));
}

// ---- DSpine injection + ln_ffn, transfer-space loss rows ----

static bool dspine_width_ok(int64_t d) { return d > 0 && d % 128 == 0 && d <= 2048; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int ksd8_dspine_ln_fwd(const void* h, const void* zsum, const void* inj, int dtype, int64_t m,
                       int64_t d, const float* gate_bias, const float* ln_w, const float* ln_b,
                       float eps, void* h2, void* out, float* mean, float* rstd, int* status,
                       void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || !dspine_width_ok(d)) return KSD8_ERR_SHAPE;
  if (!(eps > 0.f)) return KSD8_ERR_ARG;
  if (m > 0 && (!h || !zsum || !inj || !gate_bias || !ln_w || !ln_b || !h2 || !out || !mean ||
                !rstd))
    return KSD8_ERR_ARG;
  if (m > 0 && !(aligned16(h) && aligned16(zsum) && aligned16(inj) && aligned16(h2) &&
                 aligned16(out) && aligned16(gate_bias) && aligned16(ln_w) && aligned16(ln_b)))
    return KSD8_ERR_ALIGN;
  return finish(ksd8_dspine_ln_fwd_launch(h, zsum, inj, dtype, m, d, gate_bias, ln_w, ln_b, eps,
                                          h2, out, mean, rstd, S(stream)));
}

int ksd8_dspine_ln_bwd(const void* h2, const float* mean, const float* rstd, const void* db,
                       const float* dres, const void* zsum, const void* inj, int dtype, int64_t m,
                       int64_t d, const float* gate_bias, const float* ln_w, float* dh2, void* dz,
                       void* dinj, float* partials, int64_t n_parts, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || !dspine_width_ok(d)) return KSD8_ERR_SHAPE;
  if (n_parts <= 0 || n_parts > INT32_MAX || !partials || !gate_bias || !ln_w) return KSD8_ERR_ARG;
  if (m > 0 && (!h2 || !mean || !rstd || !db || !dres || !zsum || !inj || !dh2 || !dz || !dinj))
    return KSD8_ERR_ARG;
  if (m > 0 && !(aligned16(h2) && aligned16(db) && aligned16(dres) && aligned16(zsum) &&
                 aligned16(inj) && aligned16(dh2) && aligned16(dz) && aligned16(dinj) &&
                 aligned16(partials) && aligned16(gate_bias) && aligned16(ln_w)))
    return KSD8_ERR_ALIGN;
  return finish(ksd8_dspine_ln_bwd_launch(h2, mean, rstd, db, dres, zsum, inj, dtype, m, d,
                                          gate_bias, ln_w, dh2, dz, dinj, partials, n_parts,
                                          S(stream)));
}

int ksd8_transfer_rows(const void* p, int dtype, const float* e, int64_t m, int64_t d,
                       float* norm, float* dot, float* term, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || !dspine_width_ok(d)) return KSD8_ERR_SHAPE;
  if (m > 0 && (!p || !e || !norm || !dot || !term)) return KSD8_ERR_ARG;
  if (m > 0 && !(aligned16(p) && aligned16(e))) return KSD8_ERR_ALIGN;
  return finish(ksd8_transfer_rows_launch(p, dtype, e, m, d, norm, dot, term, S(stream)));
}

int ksd8_transfer_bwd(const void* p, int dtype, const float* e, const float* norm,
                      const float* dot, int64_t m, int64_t d, float coef, const void* pgrad,
                      const float* first, int64_t t_len, void* dp, float* e_grad, int* status,
                      void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || !dspine_width_ok(d)) return KSD8_ERR_SHAPE;
  if (first && (t_len <= 0 || m % t_len != 0)) return KSD8_ERR_SHAPE;
  if (m > 0 && (!p || !e || !norm || !dot || !dp || !e_grad)) return KSD8_ERR_ARG;
  if (m > 0 && !(aligned16(p) && aligned16(e) && aligned16(dp) && aligned16(e_grad) &&
                 (!pgrad || aligned16(pgrad)) && (!first || aligned16(first))))
    return KSD8_ERR_ALIGN;
  return finish(ksd8_transfer_bwd_launch(p, dtype, e, norm, dot, m, d, coef, pgrad, first,
                                         first ? t_len : 1, dp, e_grad, S(stream)));
}

// ---- incremental Rosa matching (drafting) ----

int ksd8_rosa_decode_build(const uint64_t* kw, int64_t n_streams, int64_t nw, int64_t n_keys,
                           int max_len, uint64_t* sw, uint16_t* sj, uint16_t* blk,
                           uint64_t* smp, int64_t cap, int* status, void* stream) {
  (void)status;
  if (n_streams < 0 || nw < 0 || n_keys < 0 || cap <= 0 || cap % 64 != 0) return KSD8_ERR_SHAPE;
  if (max_len < 1 || max_len > 64) return KSD8_ERR_ARG;
  if (n_keys > nw * 64 || n_keys > cap || cap > 65536) return KSD8_ERR_SHAPE;
  if (n_streams > 0 && (!kw || !sw || !sj || !blk || !smp)) return KSD8_ERR_ARG;
  return finish(ksd8_rosa_decode_build_launch(kw, n_streams, nw, n_keys, max_len, sw, sj, blk,
                                              smp, cap, S(stream)));
}

int ksd8_rosa_decode_merge(const uint64_t* kw, int64_t n_streams, int64_t nw, int64_t n_old,
                           int64_t n_new, int max_len, const uint64_t* sw_in,
                           const uint16_t* sj_in, uint64_t* sw, uint16_t* sj, uint16_t* blk,
                           uint64_t* smp, int64_t cap, int* status, void* stream) {
  (void)status;
  if (n_streams < 0 || nw < 0 || n_old < 0 || n_new < n_old || cap <= 0 || cap % 64 != 0 ||
      cap > 65536)
    return KSD8_ERR_SHAPE;
  if (max_len < 1 || max_len > 64) return KSD8_ERR_ARG;
  if (n_new > nw * 64 || n_new > cap) return KSD8_ERR_SHAPE;
  if (n_streams > 0 && (!kw || !sw_in || !sj_in || !sw || !sj || !blk || !smp))
    return KSD8_ERR_ARG;
  if (n_streams > 0 && (sw_in == sw || sj_in == sj)) return KSD8_ERR_ARG;   // out of place
  return finish(ksd8_rosa_decode_merge_launch(kw, n_streams, nw, n_old, n_new, max_len, sw_in,
                                              sj_in, sw, sj, blk, smp, cap, S(stream)));
}

int ksd8_rosa_decode_step(const void* proj_q, const void* proj_k, const void* proj_v, int dtype,
                          int64_t contexts, int64_t streams, int64_t k_new, int64_t t0,
                          int64_t n_main, int max_len, uint64_t* qw, uint64_t* kw, uint64_t* vw,
                          int64_t nw, const uint64_t* sw, const uint16_t* sj,
                          const uint16_t* blk, const uint64_t* smp, int64_t cap,
                          const float* payload, void* out, int64_t out_cs, int out_dtype,
                          int32_t* match_len, int32_t* match_end, int64_t ml_rs,
                          const int64_t* pos, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype) || !valid_float_dtype(out_dtype)) return KSD8_ERR_DTYPE;
  if (out_cs < k_new * streams || ((match_len || match_end) && ml_rs < k_new))
    return KSD8_ERR_SHAPE;
  int64_t max_new = 0, max_main = 0, max_dwords = 0;
  ksd8_rosa_decode_limits(&max_new, &max_main, &max_dwords);
  if (contexts < 0 || streams < 0 || k_new < 1 || k_new > max_new || t0 < 0 || n_main < 0 ||
      n_main > t0 || cap <= 0 || cap % 64 != 0 || nw <= 0)
    return KSD8_ERR_SHAPE;
  if (max_len < 1 || max_len > 64) return KSD8_ERR_ARG;
  if (t0 + k_new > nw * 64 || t0 + k_new > 65536 || cap > 65536) return KSD8_ERR_SHAPE;
  const int64_t r0 = max_len - 1;
  if (n_main - r0 > max_main || n_main > cap) return KSD8_ERR_UNSUPPORTED;
  const int64_t dlo = n_main > r0 ? n_main : r0, dhi = t0 + k_new - 2;
  if (dhi >= dlo) {
    const int64_t w0 = dlo > 63 ? (dlo >> 6) - 1 : 0;
    if ((dhi >> 6) - w0 + 1 > max_dwords) return KSD8_ERR_UNSUPPORTED;  // rebuild first
  }
  if ((proj_q == nullptr) != (proj_k == nullptr) || (proj_q == nullptr) != (proj_v == nullptr))
    return KSD8_ERR_ARG;
  if (contexts * streams > 0 && (!qw || !kw || !vw || !sw || !sj || !blk || !smp || !out))
    return KSD8_ERR_ARG;
  const void* proj[3] = {proj_q, proj_k, proj_v};
  uint64_t* bits[3] = {qw, kw, vw};
  return finish(ksd8_rosa_decode_step_launch(proj, dtype, contexts, streams, k_new, t0, n_main,
                                             max_len, bits, nw, sw, sj, blk, smp, cap, payload,
                                             out,
                                             out_cs, out_dtype, match_len, match_end, ml_rs,
                                             pos, S(stream)));
}

int ksd8_rosa_payload_bwd(const void* o, const int8_t* codes, const float* gx, const void* sign,
                          int dtype, int64_t m, int64_t streams, float* partials,
                          int64_t n_parts, int* status, void* stream) {
  (void)status;
  if (!valid_float_dtype(dtype)) return KSD8_ERR_DTYPE;
  if (m < 0 || streams <= 0 || streams % 4 != 0 || streams > 2048) return KSD8_ERR_SHAPE;
  if (n_parts <= 0 || n_parts > INT32_MAX || !partials) return KSD8_ERR_ARG;
  if (m > 0 && (!o || !codes || !gx || !sign)) return KSD8_ERR_ARG;
  if (m > 0 && ((reinterpret_cast<uintptr_t>(gx) & 15) || (reinterpret_cast<uintptr_t>(codes) & 3)))
    return KSD8_ERR_ALIGN;
  return finish(ksd8_rosa_payload_bwd_launch(o, codes, gx, sign, dtype, m, streams, partials,
                                             n_parts, S(stream)));
}
