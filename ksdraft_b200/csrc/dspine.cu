// DSpine adjacent injection around its low-rank GEMMs, fused with the block's
// ln_ffn LayerNorm, and the per-layer transfer-space loss rows.
//
// Forward of one DraftBlock after the Rosa residual (ksdraft/model/block.py:40-41,
// ksdraft/model/spine.py:56-69):
//     gate = sigmoid(zsum + gate_bias)          zsum = G_q z_t + G_p p_{t-1} (one GEMM)
//     h2   = h + gate * inj                     inj  = A p_{t-1}             (one GEMM)
//     b    = LayerNorm(h2; ln_w, ln_b)           (ln_ffn, eps 1e-5)
// The low-rank GEMMs stay with cuBLAS (K = 32 / 64 / 96: HBM-bound on their M x d
// side); these kernels make the elementwise and normalisation work one pass.
//
// Arithmetic: fp32 inside, every stored tensor rounded once to the activation
// dtype T (h2 is rounded before the LayerNorm reads it, as the reference's
// module boundary does); gate_bias, ln_w and ln_b are the fp32 masters rounded
// to T first (the parameters of a T-typed module).
//
// Transfer-space loss per layer (ksdraft/train/__init__.py:80-85):
//     term_t = 1 - <p_t / max(|p_t|, 1e-12), e_t>,   e_t = normalize(E[target_t])
// and its gradient with respect to p_t, for a loss coefficient c on the sum
// of the terms: c * d/dp of the above (the F.normalize backward).
#include "common.cuh"

namespace ksd8 {

namespace {

__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 x = *reinterpret_cast<const float4*>(p);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void load4(const __half* p, float (&v)[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&x.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&x.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void store4(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 x;
  x.x = *reinterpret_cast<uint32_t*>(&a);
  x.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = x;
}
__device__ __forceinline__ void store4(__half* p, const float (&v)[4]) {
  __half2 a = __floats2half2_rn(v[0], v[1]);
  __half2 b = __floats2half2_rn(v[2], v[3]);
  uint2 x;
  x.x = *reinterpret_cast<uint32_t*>(&a);
  x.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = x;
}

// value as stored in T and read back
template <typename T> __device__ __forceinline__ float round_to(float x);
template <> __device__ __forceinline__ float round_to<float>(float x) { return x; }
template <> __device__ __forceinline__ float round_to<__nv_bfloat16>(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
template <> __device__ __forceinline__ float round_to<__half>(float x) {
  return __half2float(__float2half_rn(x));
}

__device__ __forceinline__ void load4_rounded_param(const float* p, float (&v)[4], int dt) {
  load4(p, v);
  if (dt == KSD8_BF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = round_to<__nv_bfloat16>(v[i]);
  } else if (dt == KSD8_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = round_to<__half>(v[i]);
  }
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

template <typename T> __host__ __device__ constexpr int dtype_code();
template <> __host__ __device__ constexpr int dtype_code<float>() { return KSD8_F32; }
template <> __host__ __device__ constexpr int dtype_code<__nv_bfloat16>() { return KSD8_BF16; }
template <> __host__ __device__ constexpr int dtype_code<__half>() { return KSD8_F16; }

}  // namespace

// One warp per token row; lane owns the 4 columns c * 128 + 4 * lane .. + 3 of
// each 128-column chunk c < NCH (d = 128 * NCH).
template <typename T, int NCH>
__global__ void __launch_bounds__(256) dspine_ln_fwd_kernel(
    const T* __restrict__ h, const T* __restrict__ zsum, const T* __restrict__ inj,
    const float* __restrict__ gate_bias, const float* __restrict__ ln_w,
    const float* __restrict__ ln_b, float eps, int64_t m, T* __restrict__ h2, T* __restrict__ out,
    float* __restrict__ mean_out, float* __restrict__ rstd_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= m) return;
  constexpr int D = NCH * 128;
  constexpr int DT = dtype_code<T>();
  const int64_t base = row * D;
  float v[NCH][4];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 128 + lane * 4;
    float hv[4], zv[4], iv[4], bv[4];
    load4(h + base + col, hv);
    load4(zsum + base + col, zv);
    load4(inj + base + col, iv);
    load4_rounded_param(gate_bias + col, bv, DT);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float g = sigmoidf_(zv[i] + bv[i]);
      v[c][i] = round_to<T>(hv[i] + g * iv[i]);
      s += v[c][i];
    }
    store4(h2 + base + col, v[c]);
  }
  const float mean = warp_sum(s) * (1.f / D);
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float dv = v[c][i] - mean;
      ss += dv * dv;
    }
  const float rstd = rsqrtf(warp_sum(ss) * (1.f / D) + eps);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 128 + lane * 4;
    float wv[4], bv[4], o[4];
    load4_rounded_param(ln_w + col, wv, DT);
    load4_rounded_param(ln_b + col, bv, DT);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = (v[c][i] - mean) * rstd * wv[i] + bv[i];
    store4(out + base + col, o);
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// Backward.  CTA = d / 4 threads (thread owns 4 consecutive columns), rows
// [blockIdx.x * rpc, +rpc).  Per row:
//   xhat = (h2 - mean) rstd, wdy = w db,
//   dh2  = dres + rstd (wdy - mean(wdy) - xhat mean(wdy xhat))   (LayerNorm)
//   g = sigmoid(zsum + gate_bias); dinj = dh2 g; dz = dh2 inj g (1 - g)
// and the column sums of db xhat, db and dz (ln_w, ln_b, gate_bias gradients)
// into partials[blockIdx.x][3][d], summed over CTAs by the caller.
template <typename T>
__global__ void __launch_bounds__(512) dspine_ln_bwd_kernel(
    const T* __restrict__ h2, const float* __restrict__ mean, const float* __restrict__ rstd,
    const T* __restrict__ db, const float* __restrict__ dres, const T* __restrict__ zsum,
    const T* __restrict__ inj, const float* __restrict__ gate_bias,
    const float* __restrict__ ln_w, int64_t m, int d, int64_t rpc, float* __restrict__ dh2,
    T* __restrict__ dz, T* __restrict__ dinj, float* __restrict__ partials) {
  __shared__ float2 red[2][32];
  constexpr int DT = dtype_code<T>();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  const int col = tid * 4;
  float wv[4], bv[4];
  load4_rounded_param(ln_w + col, wv, DT);
  load4_rounded_param(gate_bias + col, bv, DT);
  float pw[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f}, pg[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t r0 = (int64_t)blockIdx.x * rpc;
  const int64_t r1 = min(m, r0 + rpc);
  const float inv_d = 1.f / (float)d;
  int parity = 0;
  for (int64_t row = r0; row < r1; ++row, parity ^= 1) {
    const int64_t off = row * d + col;
    const float mu = mean[row], rs = rstd[row];
    float hv[4], gv[4], xh[4], wdy[4];
    load4(h2 + off, hv);
    load4(db + off, gv);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xh[i] = (hv[i] - mu) * rs;
      wdy[i] = wv[i] * gv[i];
      s1 += wdy[i];
      s2 += wdy[i] * xh[i];
      pw[i] += gv[i] * xh[i];
      pb[i] += gv[i];
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) red[parity][warp] = make_float2(s1, s2);
    // the remaining loads do not depend on the reduction
    float rv[4], zv[4], iv[4];
    load4(dres + off, rv);
    load4(zsum + off, zv);
    load4(inj + off, iv);
    __syncthreads();
    float c1 = 0.f, c2 = 0.f;
    for (int w = 0; w < nwarps; ++w) {
      const float2 p = red[parity][w];
      c1 += p.x;
      c2 += p.y;
    }
    c1 *= inv_d;
    c2 *= inv_d;
    float o[4], di[4], dzv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[i] = rv[i] + rs * (wdy[i] - c1 - xh[i] * c2);
      const float g = sigmoidf_(zv[i] + bv[i]);
      di[i] = o[i] * g;
      dzv[i] = o[i] * iv[i] * g * (1.f - g);
      pg[i] += round_to<T>(dzv[i]);
    }
    store4(dh2 + off, o);
    store4(dinj + off, di);
    store4(dz + off, dzv);
    // red[parity] is rewritten two rows later, after the next row's barrier
  }
  float* pp = partials + (int64_t)blockIdx.x * 3 * d + col;
  store4(pp, pw);
  store4(pp + d, pb);
  store4(pp + 2 * d, pg);
}

// Transfer-space loss rows: norm_out[t] = |p_t|, dot_out[t] = <p_t, e_t>,
// term_out[t] = 1 - dot / max(|p_t|, 1e-12).  One warp per row.
template <typename T, int NCH>
__global__ void __launch_bounds__(256) transfer_rows_kernel(const T* __restrict__ p,
                                                            const float* __restrict__ e,
                                                            int64_t m, float* __restrict__ norm_out,
                                                            float* __restrict__ dot_out,
                                                            float* __restrict__ term_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= m) return;
  constexpr int D = NCH * 128;
  const int64_t base = row * D;
  float nn = 0.f, dt = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 128 + lane * 4;
    float pv[4], ev[4];
    load4(p + base + col, pv);
    load4(e + base + col, ev);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      nn += pv[i] * pv[i];
      dt += pv[i] * ev[i];
    }
  }
  nn = sqrtf(warp_sum(nn));
  dt = warp_sum(dt);
  if (lane == 0) {
    norm_out[row] = nn;
    dot_out[row] = dt;
    term_out[row] = 1.f - dt / fmaxf(nn, 1e-12f);
  }
}

// Gradient of coef * sum_t term_t with respect to p_t (and to e_t):
//   n = p / s, s = max(|p|, 1e-12):  dp = -coef (e - <e, n> n) / s   (|p| > 1e-12)
//                                    dp = -coef e / 1e-12            (clamped)
//   de -= coef n   (accumulated into e_grad)
// plus the addends pgrad (T, optional) and first[b] on the rows t % t_len == 0
// (fp32 (B, d), optional).  dp is written in T.
template <typename T, int NCH>
__global__ void __launch_bounds__(256) transfer_bwd_kernel(
    const T* __restrict__ p, const float* __restrict__ e, const float* __restrict__ norm,
    const float* __restrict__ dot, int64_t m, float coef, const T* __restrict__ pgrad,
    const float* __restrict__ first, int64_t t_len, T* __restrict__ dp,
    float* __restrict__ e_grad) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= m) return;
  constexpr int D = NCH * 128;
  const int64_t base = row * D;
  const float nrm = norm[row];
  const bool clamped = nrm <= 1e-12f;
  const float s = fmaxf(nrm, 1e-12f);
  const float en = dot[row] / s;  // <e, n>
  const float* fr = (first && row % t_len == 0) ? first + (row / t_len) * D : nullptr;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 128 + lane * 4;
    float pv[4], ev[4], gv[4], o[4];
    load4(p + base + col, pv);
    load4(e + base + col, ev);
    load4(e_grad + base + col, gv);
    float ad[4] = {0.f, 0.f, 0.f, 0.f};
    if (pgrad) load4(pgrad + base + col, ad);
    float fv[4] = {0.f, 0.f, 0.f, 0.f};
    if (fr) load4(fr + col, fv);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float n = pv[i] / s;
      const float g = clamped ? -coef * ev[i] / 1e-12f : -coef * (ev[i] - en * n) / s;
      o[i] = g + ad[i] + fv[i];
      gv[i] -= coef * n;
    }
    store4(dp + base + col, o);
    store4(e_grad + base + col, gv);
  }
}

namespace {

template <typename T, int NCH>
int launch_fwd_t(const void* h, const void* z, const void* inj, const float* gb, const float* w,
                 const float* b, float eps, int64_t m, void* h2, void* out, float* mean,
                 float* rstd, cudaStream_t st) {
  const unsigned grid = (unsigned)((m + 7) / 8);
  dspine_ln_fwd_kernel<T, NCH><<<grid, 256, 0, st>>>(
      (const T*)h, (const T*)z, (const T*)inj, gb, w, b, eps, m, (T*)h2, (T*)out, mean, rstd);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

template <typename T, int NCH>
int launch_rows_t(const void* p, const float* e, int64_t m, float* nrm, float* dot, float* term,
                  cudaStream_t st) {
  transfer_rows_kernel<T, NCH><<<(unsigned)((m + 7) / 8), 256, 0, st>>>((const T*)p, e, m, nrm,
                                                                       dot, term);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

template <typename T, int NCH>
int launch_tbwd_t(const void* p, const float* e, const float* nrm, const float* dot, int64_t m,
                  float coef, const void* pgrad, const float* first, int64_t t_len, void* dp,
                  float* eg, cudaStream_t st) {
  transfer_bwd_kernel<T, NCH><<<(unsigned)((m + 7) / 8), 256, 0, st>>>(
      (const T*)p, e, nrm, dot, m, coef, (const T*)pgrad, first, t_len, (T*)dp, eg);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

// d = 128 * nch, nch in 1..16, dispatched to a compile-time width
template <template <typename, int> class F, typename T, typename... A>
int by_width(int nch, A... args) {
  switch (nch) {
#define KSD8_W(n) \
  case n:         \
    return F<T, n>::run(args...);
    KSD8_W(1) KSD8_W(2) KSD8_W(3) KSD8_W(4) KSD8_W(5) KSD8_W(6) KSD8_W(7) KSD8_W(8)
    KSD8_W(9) KSD8_W(10) KSD8_W(11) KSD8_W(12) KSD8_W(13) KSD8_W(14) KSD8_W(15) KSD8_W(16)
#undef KSD8_W
    default:
      return KSD8_ERR_UNSUPPORTED;
  }
}

template <typename T, int NCH> struct FwdF {
  template <typename... A> static int run(A... a) { return launch_fwd_t<T, NCH>(a...); }
};
template <typename T, int NCH> struct RowsF {
  template <typename... A> static int run(A... a) { return launch_rows_t<T, NCH>(a...); }
};
template <typename T, int NCH> struct TbwdF {
  template <typename... A> static int run(A... a) { return launch_tbwd_t<T, NCH>(a...); }
};

template <template <typename, int> class F, typename... A>
int by_dtype(int dtype, int nch, A... args) {
  switch (dtype) {
    case KSD8_F32: return by_width<F, float>(nch, args...);
    case KSD8_BF16: return by_width<F, __nv_bfloat16>(nch, args...);
    case KSD8_F16: return by_width<F, __half>(nch, args...);
    default: return KSD8_ERR_DTYPE;
  }
}

}  // namespace

}  // namespace ksd8

using namespace ksd8;

int ksd8_dspine_ln_fwd_launch(const void* h, const void* zsum, const void* inj, int dtype,
                              int64_t m, int64_t d, const float* gate_bias, const float* ln_w,
                              const float* ln_b, float eps, void* h2, void* out, float* mean,
                              float* rstd, cudaStream_t stream) {
  if (m == 0) return KSD8_OK;
  return by_dtype<FwdF>(dtype, (int)(d / 128), h, zsum, inj, gate_bias, ln_w, ln_b, eps, m, h2,
                        out, mean, rstd, stream);
}

int ksd8_dspine_ln_bwd_launch(const void* h2, const float* mean, const float* rstd,
                              const void* db, const float* dres, const void* zsum,
                              const void* inj, int dtype, int64_t m, int64_t d,
                              const float* gate_bias, const float* ln_w, float* dh2, void* dz,
                              void* dinj, float* partials, int64_t n_parts,
                              cudaStream_t stream) {
  if (n_parts <= 0) return KSD8_ERR_ARG;
  const int64_t rpc = (m + n_parts - 1) / n_parts;
  const unsigned grid = (unsigned)n_parts;
  const unsigned threads = (unsigned)(d / 4);
#define KSD8_BWD(T)                                                                         \
  dspine_ln_bwd_kernel<T><<<grid, threads, 0, stream>>>(                                   \
      (const T*)h2, mean, rstd, (const T*)db, dres, (const T*)zsum, (const T*)inj, gate_bias, \
      ln_w, m, (int)d, rpc, dh2, (T*)dz, (T*)dinj, partials)
  switch (dtype) {
    case KSD8_F32: KSD8_BWD(float); break;
    case KSD8_BF16: KSD8_BWD(__nv_bfloat16); break;
    case KSD8_F16: KSD8_BWD(__half); break;
    default: return KSD8_ERR_DTYPE;
  }
#undef KSD8_BWD
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

int ksd8_transfer_rows_launch(const void* p, int dtype, const float* e, int64_t m, int64_t d,
                              float* norm, float* dot, float* term, cudaStream_t stream) {
  if (m == 0) return KSD8_OK;
  return by_dtype<RowsF>(dtype, (int)(d / 128), p, e, m, norm, dot, term, stream);
}

int ksd8_transfer_bwd_launch(const void* p, int dtype, const float* e, const float* norm,
                             const float* dot, int64_t m, int64_t d, float coef,
                             const void* pgrad, const float* first, int64_t t_len, void* dp,
                             float* e_grad, cudaStream_t stream) {
  if (m == 0) return KSD8_OK;
  return by_dtype<TbwdF>(dtype, (int)(d / 128), p, e, norm, dot, m, coef, pgrad, first, t_len,
                         dp, e_grad, stream);
}
