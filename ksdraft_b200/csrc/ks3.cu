// Fused KS3 cell kernels (ksdraft/kernels/ks3_int8.py).
//
//  ks3_pack_kernel         _repack_masters' small tensors (:262-277): spine rows
//                          packed one GS group per 6-coefficient row (pack_spine :87),
//                          warp scale softplus(.)+1e-4 / shift 0.5*tanh(.) quantised
//                          one element per group.
//  ks3_spine_quant_kernel  composed _spine_features (:169-234) on the fp16
//                          coordinates, then quantize_last_dim(h) along charts.
//  ks3_vjp_kernel          the fp16 geometry VJP of _KS3Int8Train.backward
//                          (:354-402): dc quantised along charts and along tokens,
//                          plus per-tile column partial sums of the eight
//                          coefficient / warp-scalar gradients.
//  ks3_vjp_reduce_kernel   fixed-order reduction of those partials, fp16 rounding
//                          and the STE factors (:381-395).
//
// The reference evaluates the cell in torch CPU fp16: every elementwise op is
// computed in fp32 and rounded to fp16.  The kernels below carry fp16 values
// in fp32 registers and apply exactly that rounding after each op (hmul /
// hadd / hsub); no FMA contraction is allowed on these paths.
#include "common.cuh"

namespace ksd8 {

__device__ __forceinline__ float hr(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ float hmul(float a, float b) { return hr(__fmul_rn(a, b)); }
__device__ __forceinline__ float hadd(float a, float b) { return hr(__fadd_rn(a, b)); }
__device__ __forceinline__ float hsub(float a, float b) { return hr(__fsub_rn(a, b)); }

// _round_div127 (ks3_int8.py:57-66): truncating division, then the +-63
// remainder correction.
__device__ __forceinline__ int round_div127(int v) {
  const int q = v / 127;
  const int r = v - q * 127;
  return q + (r > 63 ? 1 : (r < -63 ? -1 : 0));
}

// _lut_index (ks3_int8.py:69-72) of an fp16 value: clamp to +-3.2 (no fp16
// lies strictly between fp16(3.2) and 3.2, so the fp16 bound is exact),
// scale by 127/3.2 = 39.6875 with fp16 rounding, round half to even.
__device__ __forceinline__ int lut_index(float v16) {
  const float c = fminf(fmaxf(v16, -3.19921875f), 3.19921875f);
  return (int)rintf(hr(__fmul_rn(c, 39.6875f)));
}

__device__ __forceinline__ int lut_at(const int8_t* lut, int idx) {
  idx += 128;
  idx = idx < 0 ? 0 : (idx > 255 ? 255 : idx);
  return (int)lut[idx];
}

struct ChartParams {
  int c[6];      // spine codes
  float ps;      // packed row scale (fp16 value)
  float scale;   // warp scale in the mode's arithmetic domain
  float shift;   // warp shift
};

// Dequantised warp scalar i (code * fp16 scale, exact in fp32), rounded to
// fp16 for the fp16 arithmetic domain.  With codes == nullptr, `scales`
// already holds the dequantised fp16 values (project_fused's interface).
__device__ __forceinline__ float dequant_scalar(const int8_t* codes, const __half* scales, int64_t i,
                                                bool to_f16) {
  if (!codes) return __half2float(scales[i]);
  const float v = (float)codes[i] * __half2float(scales[i]);
  return to_f16 ? hr(v) : v;
}

// ---------------------------------------------------------------- forward spine

// NL == 2 ('int8', default) composed path.
__device__ __forceinline__ float spine_int8(float x, const ChartParams& p, const int8_t* lut) {
  const int ti = lut_index(hr(__fmul_rn(x, 0.25f)));
  const int tq = lut_at(lut, ti);
  // warp = fp16(scale16 * fp16(fp16(tq * (4/127)) + shift16))
  const float w1 = hmul((float)tq, 0.031496062874794006f);  // fp32(4/127)
  const float w2 = hadd(w1, p.shift);
  const float warp = hmul(p.scale, w2);
  const int zq = lut_at(lut, lut_index(warp));
  const int c0 = p.c[0], c1 = p.c[1], c2 = p.c[2], c3 = p.c[3], c4 = p.c[4], c5 = p.c[5];
  const int a = 2 * c0 - 2 * c1 + c2 + c3;
  const int b = -3 * c0 + 3 * c1 - 2 * c2 - c3;
  int poly = a * 64;
  poly = round_div127(poly * tq * 4) + b * 64;
  poly = round_div127(poly * tq * 4) + c2 * 64;
  poly = round_div127(poly * tq * 4) + c0 * 64;
  int warped = 4 * c5 * 64;
  warped = round_div127(warped * zq) + 2 * c4 * 64;
  warped = round_div127(warped * zq) - 3 * c5 * 64;
  warped = round_div127(warped * zq) - c4 * 64;
  const int tsum = (poly + warped) / 64;  // torch.div(..., rounding_mode="trunc")
  const float prod = hmul(hr((float)tsum), p.ps);
  float h = __fadd_rn(x, prod);
  h = fmaxf(h, 0.f);
  // per-element requantisation of the ReLU output (rank-1 amax over one value)
  float pre = __fdiv_rn(h, 127.0f);
  pre = hr(fminf(fmaxf(pre, 5.9604644775390625e-08f), 65504.0f));
  float q = fminf(fmaxf(rintf(__fdiv_rn(h, pre)), -127.f), 127.f);
  q = fmaxf(q, 0.f);
  const float sq = hmul(q, q);
  return __fmul_rn(sq, __fmul_rn(pre, pre));
}

// NL == 1 ('fp16') composed path (ks3_int8.py:186-203).
__device__ __forceinline__ float spine_fp16(float x, const ChartParams& p) {
  const float th = hr(__fmul_rn(x, 0.25f));
  const float t = hr(__fmul_rn(4.0f, tanhf(th)));
  const float warp = hr(__fmul_rn(p.scale, __fadd_rn(t, p.shift)));
  const float z = hr(tanhf(warp));
  const float c0 = (float)p.c[0], c1 = (float)p.c[1], c2 = (float)p.c[2];
  const float c3 = (float)p.c[3], c4 = (float)p.c[4], c5 = (float)p.c[5];
  const float a = hr(2.f * c0 - 2.f * c1 + c2 + c3);  // exact integers
  const float b = hr(-3.f * c0 + 3.f * c1 - 2.f * c2 - c3);
  float poly = hadd(hmul(a, t), b);
  poly = hadd(hmul(poly, t), hr(c2));
  poly = hadd(hmul(poly, t), hr(c0));
  float warped = hadd(hmul(hr(4.f * c5), z), hr(2.f * c4));
  warped = hsub(hmul(warped, z), hr(3.f * c5));
  warped = hsub(hmul(warped, z), hr(c4));
  const float s = __fmul_rn(__fadd_rn(poly, warped), p.ps);
  const float h = fmaxf(hr(__fadd_rn(x, s)), 0.f);
  return hmul(h, h);
}

// NL == 0 ('fp32') path (ks3_int8.py:172-184).
__device__ __forceinline__ float spine_fp32(float x, const ChartParams& p) {
  const float t = __fmul_rn(4.0f, tanhf(__fmul_rn(x, 0.25f)));
  const float z = tanhf(__fmul_rn(p.scale, __fadd_rn(t, p.shift)));
  const float c0 = (float)p.c[0], c1 = (float)p.c[1], c2 = (float)p.c[2];
  const float c3 = (float)p.c[3], c4 = (float)p.c[4], c5 = (float)p.c[5];
  const float a = 2.f * c0 - 2.f * c1 + c2 + c3;
  const float b = -3.f * c0 + 3.f * c1 - 2.f * c2 - c3;
  float poly = __fadd_rn(__fmul_rn(a, t), b);
  poly = __fadd_rn(__fmul_rn(poly, t), c2);
  poly = __fadd_rn(__fmul_rn(poly, t), c0);
  float warped = __fadd_rn(__fmul_rn(4.f * c5, z), 2.f * c4);
  warped = __fsub_rn(__fmul_rn(warped, z), 3.f * c5);
  warped = __fsub_rn(__fmul_rn(warped, z), c4);
  float h = __fadd_rn(x, __fmul_rn(__fadd_rn(poly, warped), p.ps));
  h = fmaxf(h, 0.f);
  return __fmul_rn(h, h);
}

struct SpineArgs {
  const __half* coords;
  int64_t m, charts;
  const int8_t* spine_codes;
  const __half* spine_scale;
  const int8_t* ws_codes;
  const __half* ws_scales;
  const int8_t* wh_codes;
  const __half* wh_scales;
  const int8_t* lut;
  int nl;
  int8_t* h_codes;
  __half* h_scales;
};

// grid.x = chart groups, grid.y = row blocks; each warp walks rows, each lane
// owns 4 consecutive charts of the group (loaded once).
__global__ void __launch_bounds__(256) ks3_spine_quant_kernel(SpineArgs a) {
  __shared__ int8_t s_lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) s_lut[i] = a.lut[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t g = blockIdx.x;
  const int64_t groups = (a.charts + 127) / 128;
  const int64_t cbase = g * 128 + lane * 4;
  ChartParams p[4];
  const bool to_f16 = a.nl != KSD8_NL_FP32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = cbase + i;
    if (c < a.charts) {
#pragma unroll
      for (int k = 0; k < 6; ++k) p[i].c[k] = a.spine_codes[c * 6 + k];
      p[i].ps = __half2float(a.spine_scale[c]);
      p[i].scale = dequant_scalar(a.ws_codes, a.ws_scales, c, to_f16);
      p[i].shift = dequant_scalar(a.wh_codes, a.wh_scales, c, to_f16);
    } else {
#pragma unroll
      for (int k = 0; k < 6; ++k) p[i].c[k] = 0;
      p[i].ps = 0.f; p[i].scale = 0.f; p[i].shift = 0.f;
    }
  }
  const int64_t rows_per_block = (a.m + gridDim.y - 1) / gridDim.y;
  const int64_t r_begin = blockIdx.y * rows_per_block;
  const int64_t r_end = min(a.m, r_begin + rows_per_block);
  for (int64_t r = r_begin + warp; r < r_end; r += 8) {
    const __half* crow = a.coords + r * a.charts;
    float h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t c = cbase + i;
      if (c < a.charts) {
        const float x = __half2float(crow[c]);
        h[i] = a.nl == KSD8_NL_INT8 ? spine_int8(x, p[i], s_lut)
               : a.nl == KSD8_NL_FP16 ? spine_fp16(x, p[i])
                                      : spine_fp32(x, p[i]);
      } else {
        h[i] = 0.f;
      }
    }
    float mx = fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3])));
    mx = warp_max(mx);
    __half sh;
    const float scale = gs_scale(mx, &sh);
    int8_t* out = a.h_codes + r * a.charts + cbase;
    if (cbase + 4 <= a.charts && ((reinterpret_cast<uintptr_t>(out) & 3) == 0)) {
      *reinterpret_cast<char4*>(out) =
          make_char4((char)gs_code(h[0], scale), (char)gs_code(h[1], scale),
                     (char)gs_code(h[2], scale), (char)gs_code(h[3], scale));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (cbase + i < a.charts) out[i] = (int8_t)gs_code(h[i], scale);
    }
    if (lane == 0) a.h_scales[r * groups + g] = sh;
  }
}

// ---------------------------------------------------------------- pack

__device__ __forceinline__ float softplus_f32(float x) {
  // torch.nn.functional.softplus, beta = 1, threshold = 20
  return x > 20.f ? x : log1pf(expf(x));
}

__global__ void ks3_pack_kernel(const float* coeffs, const float* raw_scale,
                                const float* raw_shift, int64_t charts, int8_t* spine_codes,
                                __half* spine_scale, int8_t* ws_codes, __half* ws_scales,
                                int8_t* wh_codes, __half* wh_scales) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= charts) return;
  float v[6];
  float m = 0.f;
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    v[k] = coeffs[c * 6 + k];
    m = fmaxf(m, fabsf(v[k]));
  }
  __half sh;
  float s = gs_scale(m, &sh);
#pragma unroll
  for (int k = 0; k < 6; ++k) spine_codes[c * 6 + k] = (int8_t)gs_code(v[k], s);
  spine_scale[c] = sh;
  const float sc = __fadd_rn(softplus_f32(raw_scale[c]), 9.99999974737875e-05f);  // + fp32(1e-4)
  s = gs_scale(fabsf(sc), &sh);
  ws_codes[c] = (int8_t)gs_code(sc, s);
  ws_scales[c] = sh;
  const float sf = __fmul_rn(0.5f, tanhf(raw_shift[c]));
  s = gs_scale(fabsf(sf), &sh);
  wh_codes[c] = (int8_t)gs_code(sf, s);
  wh_scales[c] = sh;
}

// ---------------------------------------------------------------- backward VJP

struct VjpArgs {
  const __half* value;
  const __half* coords;
  int64_t m, charts;
  const int8_t* spine_codes;
  const __half* spine_scale;
  const int8_t* ws_codes;
  const __half* ws_scales;
  const int8_t* wh_codes;
  const __half* wh_scales;
  int8_t* dc_codes;
  __half* dc_scales;
  int8_t* dct_codes;
  __half* dct_scales;
  float* partials;
};

struct VjpChart {
  float c0, c1, c2, c4, c5;
  float cubic, quad, cubic3, quad2, c5x4, c4x2, c5x12, c4x4, c5x3;
  float scale, shift;
};

constexpr int VJP_TM = 128;  // token rows per CTA (= one token-quantisation group)
constexpr int VJP_TC = 128;  // charts per CTA (= one chart-quantisation group)
constexpr int VJP_LD = VJP_TC + 1;
constexpr int VJP_SMEM = (VJP_TM * VJP_LD + 8 * 8 * VJP_TC) * 4;

__global__ void __launch_bounds__(256) ks3_vjp_kernel(VjpArgs a) {
  extern __shared__ float vsm[];
  float* tile = vsm;                       // [VJP_TM][VJP_LD] dc values
  float* red = vsm + VJP_TM * VJP_LD;      // [8 warps][8 sums][VJP_TC]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t m0 = (int64_t)blockIdx.y * VJP_TM;
  const int64_t cg = blockIdx.x;           // chart group
  const int64_t cbase = cg * VJP_TC + lane * 4;

  VjpChart ch[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t c = cbase + i;
    const float ps = __half2float(a.spine_scale[c]);
    float cc[6];
#pragma unroll
    for (int k = 0; k < 6; ++k) cc[k] = hr((float)a.spine_codes[c * 6 + k] * ps);
    VjpChart& q = ch[i];
    q.c0 = cc[0]; q.c1 = cc[1]; q.c2 = cc[2]; q.c4 = cc[4]; q.c5 = cc[5];
    // cubic = 2*c0 - 2*c1 + c2 + c3 ; quad = -3*c0 + 3*c1 - 2*c2 - c3 (fp16 ops, left to right)
    q.cubic = hadd(hadd(hsub(hmul(2.f, cc[0]), hmul(2.f, cc[1])), cc[2]), cc[3]);
    q.quad = hsub(hsub(hadd(hmul(-3.f, cc[0]), hmul(3.f, cc[1])), hmul(2.f, cc[2])), cc[3]);
    q.cubic3 = hmul(3.f, q.cubic);
    q.quad2 = hmul(2.f, q.quad);
    q.c5x4 = hmul(4.f, cc[5]);
    q.c4x2 = hmul(2.f, cc[4]);
    q.c5x12 = hmul(12.f, cc[5]);
    q.c4x4 = hmul(4.f, cc[4]);
    q.c5x3 = hmul(3.f, cc[5]);
    q.scale = dequant_scalar(a.ws_codes, a.ws_scales, c, true);
    q.shift = dequant_scalar(a.wh_codes, a.wh_scales, c, true);
  }

  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[i][k] = 0.f;

  const int64_t gcharts = a.charts / 128;
  for (int rr = warp; rr < VJP_TM; rr += 8) {
    const int64_t r = m0 + rr;
    float dc[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < a.m) {
      const uint2 vv = *reinterpret_cast<const uint2*>(a.value + r * a.charts + cbase);
      const uint2 xv = *reinterpret_cast<const uint2*>(a.coords + r * a.charts + cbase);
      const __half* ve = reinterpret_cast<const __half*>(&vv);
      const __half* xe = reinterpret_cast<const __half*>(&xv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const VjpChart& q = ch[i];
        const float value = __half2float(ve[i]);
        const float x16 = __half2float(xe[i]);
        const float th = hr(tanhf(hmul(x16, 0.25f)));
        const float t = hmul(4.f, th);
        const float u = hadd(t, q.shift);
        const float z = hr(tanhf(hmul(q.scale, u)));
        float sp = hadd(hmul(q.cubic, t), q.quad);
        sp = hadd(hmul(sp, t), q.c2);
        sp = hadd(hmul(sp, t), q.c0);
        float wp = hadd(hmul(q.c5x4, z), q.c4x2);
        wp = hsub(hmul(wp, z), q.c5x3);
        wp = hsub(hmul(wp, z), q.c4);
        const float rl = fmaxf(hadd(hadd(x16, sp), wp), 0.f);
        const float dpre = hmul(hmul(value, 2.f), rl);
        float dpoly = hadd(hmul(q.cubic3, t), q.quad2);
        dpoly = hadd(hmul(dpoly, t), q.c2);
        float dwarp = hadd(hmul(q.c5x12, z), q.c4x4);
        dwarp = hsub(hmul(dwarp, z), q.c5x3);
        const float zz = hmul(z, z);
        const float dz = hmul(dwarp, hsub(1.f, zz));
        const float tt = hmul(t, t);
        const float dmean = hmul(hmul(dpre, hadd(dpoly, hmul(dz, q.scale))),
                                 hsub(1.f, hmul(tt, 0.0625f)));
        dc[i] = hadd(value, dmean);
        const float t3 = hmul(tt, t);
        const float z3 = hmul(zz, z);
        acc[i][0] += hmul(dpre, hadd(hsub(hmul(2.f, t3), hmul(3.f, tt)), 1.f));
        acc[i][1] += hmul(dpre, hadd(hmul(-2.f, t3), hmul(3.f, tt)));
        acc[i][2] += hmul(dpre, hadd(hsub(t3, hmul(2.f, tt)), t));
        acc[i][3] += hmul(dpre, hsub(t3, tt));
        acc[i][4] += hmul(dpre, hsub(hmul(2.f, zz), 1.f));
        acc[i][5] += hmul(dpre, hsub(hmul(4.f, z3), hmul(3.f, z)));
        const float dd = hmul(dpre, dz);
        acc[i][6] += hmul(dd, u);
        acc[i][7] += hmul(dd, q.scale);
      }
      // dc quantised along charts: this row's 128 charts are one group.
      float mx = fmaxf(fmaxf(fabsf(dc[0]), fabsf(dc[1])), fmaxf(fabsf(dc[2]), fabsf(dc[3])));
      mx = warp_max(mx);
      __half sh;
      const float s = gs_scale(mx, &sh);
      *reinterpret_cast<char4*>(a.dc_codes + r * a.charts + cbase) =
          make_char4((char)gs_code(dc[0], s), (char)gs_code(dc[1], s), (char)gs_code(dc[2], s),
                     (char)gs_code(dc[3], s));
      if (lane == 0) a.dc_scales[r * gcharts + cg] = sh;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) tile[rr * VJP_LD + lane * 4 + i] = dc[i];
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 8; ++k) red[(warp * 8 + k) * VJP_TC + lane * 4 + i] = acc[i][k];
  __syncthreads();

  // dc^T quantised along tokens: column c of the tile is one group of 128 tokens.
  const int64_t mgroups = (a.m + 127) / 128;
  for (int cc = warp; cc < VJP_TC; cc += 8) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = tile[(lane + 32 * i) * VJP_LD + cc];
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    mx = warp_max(mx);
    __half sh;
    const float s = gs_scale(mx, &sh);
    const int64_t c = cg * VJP_TC + cc;
    int8_t* out = a.dct_codes + c * a.m + m0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (m0 + lane + 32 * i < a.m) out[lane + 32 * i] = (int8_t)gs_code(v[i], s);
    if (lane == 0) a.dct_scales[c * mgroups + blockIdx.y] = sh;
  }
  // Column partials: fixed-order sum over the 8 warps.
  for (int idx = threadIdx.x; idx < 8 * VJP_TC; idx += blockDim.x) {
    const int k = idx / VJP_TC, cc = idx % VJP_TC;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[(w * 8 + k) * VJP_TC + cc];
    a.partials[((int64_t)blockIdx.y * 8 + k) * a.charts + cg * VJP_TC + cc] = s;
  }
}

__global__ void ks3_vjp_reduce_kernel(const float* partials, int64_t n_tiles, int64_t charts,
                                      const float* raw_scale, const float* raw_shift,
                                      __half* dcoeff, __half* dscale, __half* dshift,
                                      int* status) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= charts) return;
  float s[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) s[k] = 0.f;
  for (int64_t t = 0; t < n_tiles; ++t)
#pragma unroll
    for (int k = 0; k < 8; ++k) s[k] += partials[(t * 8 + k) * charts + c];
  bool bad = false;
#pragma unroll
  for (int k = 0; k < 6; ++k) {
    const __half h = __float2half_rn(s[k]);
    bad |= __hisinf(h) || __hisnan(h);
    dcoeff[c * 6 + k] = h;
  }
  const float sig = 1.f / (1.f + expf(-raw_scale[c]));
  const float th = tanhf(raw_shift[c]);
  const float dscale_t = hr(s[6]);
  const float dshift_t = hmul(hr(s[7]), 0.5f);
  const __half ds = __float2half_rn(__fmul_rn(dscale_t, sig));
  const __half dh = __float2half_rn(__fmul_rn(dshift_t, __fsub_rn(1.f, __fmul_rn(th, th))));
  bad |= __hisinf(ds) || __hisnan(ds) || __hisinf(dh) || __hisnan(dh);
  dscale[c] = ds;
  dshift[c] = dh;
  if (bad) record_error(status, KSD8_ERR_NONFINITE);
}

}  // namespace ksd8

using namespace ksd8;

int ksd8_ks3_pack_launch(const float* coeffs, const float* raw_scale, const float* raw_shift,
                         int64_t charts, int8_t* spine_codes, void* spine_scale, int8_t* ws_codes,
                         void* ws_scales, int8_t* wh_codes, void* wh_scales, cudaStream_t stream) {
  if (charts == 0) return KSD8_OK;
  ks3_pack_kernel<<<(unsigned)((charts + 255) / 256), 256, 0, stream>>>(
      coeffs, raw_scale, raw_shift, charts, spine_codes, reinterpret_cast<__half*>(spine_scale),
      ws_codes, reinterpret_cast<__half*>(ws_scales), wh_codes,
      reinterpret_cast<__half*>(wh_scales));
  return KSD8_OK;
}

int ksd8_ks3_spine_quant_launch(const void* coords, int64_t m, int64_t charts,
                                const int8_t* spine_codes, const void* spine_scale,
                                const int8_t* ws_codes, const void* ws_scales,
                                const int8_t* wh_codes, const void* wh_scales, const int8_t* lut,
                                int nl, int8_t* h_codes, void* h_scales, cudaStream_t stream) {
  if (m == 0 || charts == 0) return KSD8_OK;
  SpineArgs a;
  a.coords = reinterpret_cast<const __half*>(coords);
  a.m = m; a.charts = charts; a.spine_codes = spine_codes;
  a.spine_scale = reinterpret_cast<const __half*>(spine_scale);
  a.ws_codes = ws_codes; a.ws_scales = reinterpret_cast<const __half*>(ws_scales);
  a.wh_codes = wh_codes; a.wh_scales = reinterpret_cast<const __half*>(wh_scales);
  a.lut = lut; a.nl = nl; a.h_codes = h_codes; a.h_scales = reinterpret_cast<__half*>(h_scales);
  const int64_t groups = (charts + 127) / 128;
  int64_t yb = (148 * 8 + groups - 1) / groups;  // ~8 CTAs per SM in total
  const int64_t max_yb = (m + 7) / 8;
  if (yb > max_yb) yb = max_yb;
  if (yb < 1) yb = 1;
  dim3 grid((unsigned)groups, (unsigned)yb);
  ks3_spine_quant_kernel<<<grid, 256, 0, stream>>>(a);
  return KSD8_OK;
}

int ksd8_ks3_vjp_launch(const void* value, const void* coords, int64_t m, int64_t charts,
                        const int8_t* spine_codes, const void* spine_scale, const int8_t* ws_codes,
                        const void* ws_scales, const int8_t* wh_codes, const void* wh_scales,
                        int8_t* dc_codes, void* dc_scales, int8_t* dct_codes, void* dct_scales,
                        float* partials, cudaStream_t stream) {
  if (m == 0) return KSD8_OK;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << dev))) {
    if (cudaFuncSetAttribute(ks3_vjp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             VJP_SMEM) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    attr_dev_mask |= (1 << dev);
  }
  VjpArgs a;
  a.value = reinterpret_cast<const __half*>(value);
  a.coords = reinterpret_cast<const __half*>(coords);
  a.m = m; a.charts = charts; a.spine_codes = spine_codes;
  a.spine_scale = reinterpret_cast<const __half*>(spine_scale);
  a.ws_codes = ws_codes; a.ws_scales = reinterpret_cast<const __half*>(ws_scales);
  a.wh_codes = wh_codes; a.wh_scales = reinterpret_cast<const __half*>(wh_scales);
  a.dc_codes = dc_codes; a.dc_scales = reinterpret_cast<__half*>(dc_scales);
  a.dct_codes = dct_codes; a.dct_scales = reinterpret_cast<__half*>(dct_scales);
  a.partials = partials;
  dim3 grid((unsigned)(charts / VJP_TC), (unsigned)((m + VJP_TM - 1) / VJP_TM));
  ks3_vjp_kernel<<<grid, 256, VJP_SMEM, stream>>>(a);
  return KSD8_OK;
}

int ksd8_ks3_vjp_reduce_launch(const float* partials, int64_t n_tiles, int64_t charts,
                               const float* raw_scale, const float* raw_shift, void* dcoeff16,
                               void* dscale16, void* dshift16, int* status, cudaStream_t stream) {
  if (charts == 0) return KSD8_OK;
  ks3_vjp_reduce_kernel<<<(unsigned)((charts + 127) / 128), 128, 0, stream>>>(
      partials, n_tiles, charts, raw_scale, raw_shift, reinterpret_cast<__half*>(dcoeff16),
      reinterpret_cast<__half*>(dscale16), reinterpret_cast<__half*>(dshift16), status);
  return KSD8_OK;
}
