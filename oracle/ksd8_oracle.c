/*
 * ksd8_oracle.c — CPU restatement of KSDraft's INT8 hot path (TEST
 * INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py as the checker and the CPU
 * baseline; never linked into, or called by, the ksdraft_b200 product path).
 *
 * Each function restates the reference algorithm (paths within
 * curvedinf/ksdraft) in plain C; fp16 values are handled with _Float16
 * conversions (round to nearest even) and every fp16 "op" of the reference's
 * torch CPU evaluation is computed in fp32 and rounded, as torch does.
 * Build: oracle/build.py (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef uint16_t f16bits;

static inline float h2f(f16bits b) {
  _Float16 h;
  memcpy(&h, &b, 2);
  return (float)h;
}
static inline f16bits f2h(float f) {
  _Float16 h = (_Float16)f;
  f16bits b;
  memcpy(&b, &h, 2);
  return b;
}
static inline float hr(float v) { return (float)(_Float16)v; }
static inline float hmul(float a, float b) { return hr(a * b); }
static inline float hadd(float a, float b) { return hr(a + b); }
static inline float hsub(float a, float b) { return hr(a - b); }

/* fp16 tanh of an fp16 value, correctly rounded: the reference's CPU
 * torch.tanh on fp16 (ks3_int8.py:366-367) and on fp16-valued fp32 followed
 * by .to(float16) (:189-192) give exactly this for every fp16 input (the tests
 * check all of them).  double tanh, then double -> fp32 -> fp16 (an exact
 * rounding, 24 >= 2 * 11 + 2). */
static inline float tanh16r(float v16) { return hr((float)tanh((double)v16)); }

/* tanh16r over the fp16 bit patterns 0..n-1 (non-negative values). */
void or_tanh16_table(int64_t n, f16bits* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2h(tanh16r(h2f((f16bits)i)));
}

/* GS scale of quant.py:47-49: fp32 amax/127, clamp [2^-24, 65504], round via fp16. */
static inline float gs_scale(float amax, f16bits* out) {
  float s = amax / 127.0f;
  if (s < 5.9604644775390625e-08f) s = 5.9604644775390625e-08f;
  if (s > 65504.0f) s = 65504.0f;
  f16bits b = f2h(s);
  if (out) *out = b;
  return h2f(b);
}
/* code of quant.py:50: clamp(round_half_even(x/scale), -127, 127). */
static inline int gs_code(float x, float scale) {
  float q = rintf(x / scale);
  if (q < -127.f) q = -127.f;
  if (q > 127.f) q = 127.f;
  return (int)q;
}

/* ---------------------------------------------------------------- Philox4x32-10
 * Salmon et al., "Parallel random numbers: as easy as 1, 2, 3" (SC'11). */
static void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
  }
}

float or_philox_uniform1(uint64_t seed, uint64_t idx) {
  uint32_t c[4] = {(uint32_t)(idx >> 2), (uint32_t)(idx >> 34), 0u, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(c[idx & 3] >> 8) * 5.9604644775390625e-08f;
}

void or_philox_uniform(uint64_t seed, uint64_t offset, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = or_philox_uniform1(seed, offset + (uint64_t)i);
}

/* ---------------------------------------------------------------- quantisers
 * quantize_last_dim (ksdraft/kernels/quant.py:30-52) over fp32 rows, with the
 * PTQR dither of ksdraft/train/stages.py:38-48 when dither > 0 (noise U from
 * `u` if given, else Philox(seed, offset + r*Kp + c)).  round_f16: the input
 * first goes through fp16 (x.float().to(float16)). */
void or_quantize_rows(const float* x, int64_t rows, int64_t k, int round_f16, float dither,
                      uint64_t seed, uint64_t offset, const float* u, int8_t* codes,
                      f16bits* scales) {
  const int64_t G = (k + 127) / 128, kp = G * 128;
  const float d2 = 2.0f * dither;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g = 0; g < G; ++g) {
      float v[128];
      float amax = 0.f;
      for (int i = 0; i < 128; ++i) {
        int64_t c = g * 128 + i;
        float xv = c < k ? x[r * k + c] : 0.f;
        if (round_f16) xv = hr(xv);
        v[i] = xv;
        float a = fabsf(xv);
        if (a > amax) amax = a;
      }
      f16bits sb;
      float s = gs_scale(amax, &sb);
      scales[r * G + g] = sb;
      for (int i = 0; i < 128; ++i) {
        int64_t c = g * 128 + i;
        if (c >= k) break;
        int q;
        if (dither > 0.f) {
          int64_t flat = r * kp + c;
          float uu = u ? u[flat] : or_philox_uniform1(seed, offset + (uint64_t)flat);
          float t = v[i] / s + (uu - 0.5f) * d2;
          float rr = rintf(t);
          if (rr < -127.f) rr = -127.f;
          if (rr > 127.f) rr = 127.f;
          q = (int)rr;
        } else {
          q = gs_code(v[i], s);
        }
        codes[r * k + c] = (int8_t)q;
      }
    }
  }
}

/* dequantize_last_dim (quant.py:55-67): code * scale, exact in fp32. */
void or_dequantize_rows(const int8_t* codes, const f16bits* scales, int64_t rows, int64_t k,
                        float* out) {
  const int64_t G = (k + 127) / 128;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < k; ++c)
      out[r * k + c] = (float)codes[r * k + c] * h2f(scales[r * G + c / 128]);
}

/* ---------------------------------------------------------------- W8A8 GEMM
 * Per-group int32 dot products of gemm.py:34-45 and the canonical fp32 group
 * sum acc = fmaf(RN(float(dot_g) * sa), sw, acc), g = 0..G-1.  k % 128 == 0. */
void or_w8a8_gemm(const int8_t* a, const f16bits* as, const int8_t* w, const f16bits* ws,
                  int64_t m, int64_t n, int64_t k, float* out, int32_t* partials) {
  const int64_t G = k / 128;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      float acc = 0.f;
      for (int64_t g = 0; g < G; ++g) {
        const int8_t* ap = a + i * k + g * 128;
        const int8_t* wp = w + j * k + g * 128;
        int32_t dot = 0;
        for (int t = 0; t < 128; ++t) dot += (int32_t)ap[t] * (int32_t)wp[t];
        if (partials) partials[(g * m + i) * n + j] = dot;
        /* t = RN(dot * sa) ((float)dot is exact), then one fused step with sw */
        const float t = (float)dot * h2f(as[i * G + g]);
        acc = fmaf(t, h2f(ws[j * G + g]), acc);
      }
      out[i * n + j] = acc;
    }
  }
}

/* ---------------------------------------------------------------- KS3 pack
 * pack_spine (ks3_int8.py:87-92) and the warp-scalar quantisation of
 * _repack_masters (:270-275). */
void or_ks3_pack(const float* coeffs, const float* raw_scale, const float* raw_shift,
                 int64_t charts, int8_t* spine_codes, f16bits* spine_scale, int8_t* ws_codes,
                 f16bits* ws_scales, int8_t* wh_codes, f16bits* wh_scales) {
  for (int64_t c = 0; c < charts; ++c) {
    float amax = 0.f;
    for (int k = 0; k < 6; ++k) {
      float a = fabsf(coeffs[c * 6 + k]);
      if (a > amax) amax = a;
    }
    f16bits sb;
    float s = gs_scale(amax, &sb);
    for (int k = 0; k < 6; ++k) spine_codes[c * 6 + k] = (int8_t)gs_code(coeffs[c * 6 + k], s);
    spine_scale[c] = sb;
    float x = raw_scale[c];
    float sp = x > 20.f ? x : log1pf(expf(x));
    float sc = sp + 1e-4f;
    s = gs_scale(fabsf(sc), &sb);
    ws_codes[c] = (int8_t)gs_code(sc, s);
    ws_scales[c] = sb;
    float sf = 0.5f * tanhf(raw_shift[c]);
    s = gs_scale(fabsf(sf), &sb);
    wh_codes[c] = (int8_t)gs_code(sf, s);
    wh_scales[c] = sb;
  }
}

/* ---------------------------------------------------------------- KS3 spine
 * Composed _spine_features (ks3_int8.py:169-234), rank-1 charts, on fp16
 * coordinates, followed by quantize_last_dim(h) along charts.  Warp scalars
 * come as codes + fp16 scales (dequantised exactly, then rounded to fp16
 * outside the fp32 mode); nl: 0 fp32, 1 fp16, 2 int8. */

static int round_div127(int v) {
  int q = v / 127, r = v - q * 127;
  return q + (r > 63 ? 1 : (r < -63 ? -1 : 0));
}
static int lut_index(float v16) {
  float c = v16;
  if (c < -3.19921875f) c = -3.19921875f;
  if (c > 3.19921875f) c = 3.19921875f;
  return (int)rintf(hr(c * 39.6875f));
}
static int lut_at(const int8_t* lut, int i) {
  i += 128;
  if (i < 0) i = 0;
  if (i > 255) i = 255;
  return lut[i];
}

float or_spine1(float x, const int8_t* cc, float ps, float scale, float shift,
                const int8_t* lut, int nl) {
  const int c0 = cc[0], c1 = cc[1], c2 = cc[2], c3 = cc[3], c4 = cc[4], c5 = cc[5];
  if (nl == 2) {
    int ti = lut_index(hr(x * 0.25f));
    int tq = lut_at(lut, ti);
    float w1 = hmul((float)tq, (float)(4.0 / 127.0));
    float w2 = hadd(w1, shift);
    float warp = hmul(scale, w2);
    int zq = lut_at(lut, lut_index(warp));
    int a = 2 * c0 - 2 * c1 + c2 + c3;
    int b = -3 * c0 + 3 * c1 - 2 * c2 - c3;
    int poly = a * 64;
    poly = round_div127(poly * tq * 4) + b * 64;
    poly = round_div127(poly * tq * 4) + c2 * 64;
    poly = round_div127(poly * tq * 4) + c0 * 64;
    int warped = 4 * c5 * 64;
    warped = round_div127(warped * zq) + 2 * c4 * 64;
    warped = round_div127(warped * zq) - 3 * c5 * 64;
    warped = round_div127(warped * zq) - c4 * 64;
    int tsum = (poly + warped) / 64;
    float h = x + hmul(hr((float)tsum), ps);
    if (h < 0.f) h = 0.f;
    float pre = h / 127.0f;
    if (pre < 5.9604644775390625e-08f) pre = 5.9604644775390625e-08f;
    if (pre > 65504.f) pre = 65504.f;
    pre = hr(pre);
    float q = rintf(h / pre);
    if (q < -127.f) q = -127.f;
    if (q > 127.f) q = 127.f;
    if (q < 0.f) q = 0.f;
    float sq = hmul(q, q);
    return sq * (pre * pre);
  }
  if (nl == 1) {
    float th = hr(x * 0.25f);
    float t = hr(4.0f * tanh16r(th));
    float warp = hr(scale * (t + shift));
    float z = tanh16r(warp);
    float a = hr((float)(2 * c0 - 2 * c1 + c2 + c3));
    float b = hr((float)(-3 * c0 + 3 * c1 - 2 * c2 - c3));
    float poly = hadd(hmul(a, t), b);
    poly = hadd(hmul(poly, t), hr((float)c2));
    poly = hadd(hmul(poly, t), hr((float)c0));
    float warped = hadd(hmul(hr(4.f * c5), z), hr(2.f * c4));
    warped = hsub(hmul(warped, z), hr(3.f * c5));
    warped = hsub(hmul(warped, z), hr((float)c4));
    float h = hr(x + (poly + warped) * ps);
    if (h < 0.f) h = 0.f;
    return hmul(h, h);
  }
  {
    float t = 4.0f * tanhf(x * 0.25f);
    float z = tanhf(scale * (t + shift));
    float a = (float)(2 * c0 - 2 * c1 + c2 + c3);
    float b = (float)(-3 * c0 + 3 * c1 - 2 * c2 - c3);
    float poly = ((a * t + b) * t + (float)c2) * t + (float)c0;
    float warped = ((4.f * c5 * z + 2.f * c4) * z - 3.f * c5) * z - (float)c4;
    float h = x + (poly + warped) * ps;
    if (h < 0.f) h = 0.f;
    return h * h;
  }
}

static float dq_scalar(const int8_t* codes, const f16bits* scales, int64_t i, int to_f16) {
  if (!codes) return h2f(scales[i]);
  float v = (float)codes[i] * h2f(scales[i]);
  return to_f16 ? hr(v) : v;
}

void or_ks3_spine_quant(const f16bits* coords, int64_t m, int64_t charts,
                        const int8_t* spine_codes, const f16bits* spine_scale,
                        const int8_t* ws_codes, const f16bits* ws_scales, const int8_t* wh_codes,
                        const f16bits* wh_scales, const int8_t* lut, int nl, float* h_out,
                        int8_t* h_codes, f16bits* h_scales) {
  const int64_t G = (charts + 127) / 128;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    for (int64_t g = 0; g < G; ++g) {
      float h[128];
      float amax = 0.f;
      for (int i = 0; i < 128; ++i) {
        int64_t c = g * 128 + i;
        if (c >= charts) {
          h[i] = 0.f;
          continue;
        }
        float sc = dq_scalar(ws_codes, ws_scales, c, nl != 0);
        float sh = dq_scalar(wh_codes, wh_scales, c, nl != 0);
        h[i] = or_spine1(h2f(coords[r * charts + c]), spine_codes + c * 6, h2f(spine_scale[c]),
                         sc, sh, lut, nl);
        if (h_out) h_out[r * charts + c] = h[i];
        float a = fabsf(h[i]);
        if (a > amax) amax = a;
      }
      if (!h_codes) continue;
      f16bits sb;
      float s = gs_scale(amax, &sb);
      h_scales[r * G + g] = sb;
      for (int i = 0; i < 128; ++i) {
        int64_t c = g * 128 + i;
        if (c < charts) h_codes[r * charts + c] = (int8_t)gs_code(h[i], s);
      }
    }
  }
}

/* ---------------------------------------------------------------- KS3 VJP
 * Geometry VJP of _KS3Int8Train.backward (ks3_int8.py:354-402) in torch's
 * fp16 evaluation order.  Writes dc (fp32 values of the fp16 results,
 * (m, charts)) and the eight column sums (8, charts) accumulated in fp32
 * (d0..d5, dscale_t, dshift_t before its 0.5 factor). */
void or_ks3_vjp(const f16bits* value, const f16bits* coords, int64_t m, int64_t charts,
                const int8_t* spine_codes, const f16bits* spine_scale, const int8_t* ws_codes,
                const f16bits* ws_scales, const int8_t* wh_codes, const f16bits* wh_scales,
                float* dc_out, float* sums) {
  for (int64_t k = 0; k < 8 * charts; ++k) sums[k] = 0.f;
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < charts; ++c) {
    const float ps = h2f(spine_scale[c]);
    float cc[6];
    for (int k = 0; k < 6; ++k) cc[k] = hr((float)spine_codes[c * 6 + k] * ps);
    const float c0 = cc[0], c1 = cc[1], c2 = cc[2], c3 = cc[3], c4 = cc[4], c5 = cc[5];
    const float cubic = hadd(hadd(hsub(hmul(2.f, c0), hmul(2.f, c1)), c2), c3);
    const float quad = hsub(hsub(hadd(hmul(-3.f, c0), hmul(3.f, c1)), hmul(2.f, c2)), c3);
    const float scale = dq_scalar(ws_codes, ws_scales, c, 1);
    const float shift = dq_scalar(wh_codes, wh_scales, c, 1);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t r = 0; r < m; ++r) {
      const float v = h2f(value[r * charts + c]);
      const float x16 = h2f(coords[r * charts + c]);
      const float t = hmul(4.f, tanh16r(hmul(x16, 0.25f)));
      const float u = hadd(t, shift);
      const float z = tanh16r(hmul(scale, u));
      float sp = hadd(hmul(cubic, t), quad);
      sp = hadd(hmul(sp, t), c2);
      sp = hadd(hmul(sp, t), c0);
      float wp = hadd(hmul(hmul(4.f, c5), z), hmul(2.f, c4));
      wp = hsub(hmul(wp, z), hmul(3.f, c5));
      wp = hsub(hmul(wp, z), c4);
      float rl = hadd(hadd(x16, sp), wp);
      if (rl < 0.f) rl = 0.f;
      const float dpre = hmul(hmul(v, 2.f), rl);
      float dpoly = hadd(hmul(hmul(3.f, cubic), t), hmul(2.f, quad));
      dpoly = hadd(hmul(dpoly, t), c2);
      float dwarp = hadd(hmul(hmul(12.f, c5), z), hmul(4.f, c4));
      dwarp = hsub(hmul(dwarp, z), hmul(3.f, c5));
      const float zz = hmul(z, z);
      const float dz = hmul(dwarp, hsub(1.f, zz));
      const float tt = hmul(t, t);
      const float dmean =
          hmul(hmul(dpre, hadd(dpoly, hmul(dz, scale))), hsub(1.f, hmul(tt, 0.0625f)));
      dc_out[r * charts + c] = hadd(v, dmean);
      const float t3 = hmul(tt, t), z3 = hmul(zz, z);
      acc[0] += hmul(dpre, hadd(hsub(hmul(2.f, t3), hmul(3.f, tt)), 1.f));
      acc[1] += hmul(dpre, hadd(hmul(-2.f, t3), hmul(3.f, tt)));
      acc[2] += hmul(dpre, hadd(hsub(t3, hmul(2.f, tt)), t));
      acc[3] += hmul(dpre, hsub(t3, tt));
      acc[4] += hmul(dpre, hsub(hmul(2.f, zz), 1.f));
      acc[5] += hmul(dpre, hsub(hmul(4.f, z3), hmul(3.f, z)));
      const float dd = hmul(dpre, dz);
      acc[6] += hmul(dd, u);
      acc[7] += hmul(dd, scale);
    }
    for (int k = 0; k < 8; ++k) sums[k * charts + c] = acc[k];
  }
}

/* ---------------------------------------------------------------- Rosa
 * _match_payload_sign (ksdraft/model/rosa.py:40-98) by its definition: for
 * each t, lengths L from min(max_len, t) down to 1, endpoints j from t-1
 * down to L-1; the first (L, j) whose windows agree decides. */
void or_rosa_match_bruteforce(const int8_t* q, const int8_t* k, const int8_t* v, int64_t streams,
                              int64_t T, int max_len, float* sign, int32_t* mlen,
                              int32_t* mend) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t s = 0; s < streams; ++s) {
    const int8_t* qs = q + s * T;
    const int8_t* ks = k + s * T;
    const int8_t* vs = v + s * T;
    for (int64_t t = 0; t < T; ++t) {
      int64_t bestj = -1;
      int bestl = 0;
      int64_t lmax = t < max_len ? t : max_len;
      for (int64_t L = lmax; L >= 1 && bestj < 0; --L) {
        for (int64_t j = t - 1; j >= L - 1; --j) {
          int ok = 1;
          for (int64_t i = 0; i < L; ++i)
            if ((qs[t - i] > 0) != (ks[j - i] > 0)) {
              ok = 0;
              break;
            }
          if (ok) {
            bestj = j;
            bestl = (int)L;
            break;
          }
        }
      }
      sign[s * T + t] = bestj >= 0 ? (vs[bestj + 1] > 0 ? 1.f : -1.f) : -1.f;
      if (mlen) mlen[s * T + t] = bestl;
      if (mend) mend[s * T + t] = (int32_t)bestj;
    }
  }
}

/* Same result in O(T^2) per stream: run[j] = length of the common suffix of
 * q[..t] and k[..j] (uncapped, updated along diagonals), capped at
 * min(max_len, j+1); the maximum, latest j on ties.  `work` holds 2*T ints
 * per thread slot (streams processed sequentially per slot). */
void or_rosa_match_dp(const int8_t* q, const int8_t* k, const int8_t* v, int64_t streams,
                      int64_t T, int max_len, float* sign, int32_t* mlen, int32_t* mend,
                      int32_t* work, int n_slots) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(n_slots)
  for (int64_t s = 0; s < streams; ++s) {
#ifdef _OPENMP
    int32_t* run = work + (int64_t)omp_get_thread_num() * 2 * T;
#else
    int32_t* run = work;
#endif
    const int8_t* qs = q + s * T;
    const int8_t* ks = k + s * T;
    const int8_t* vs = v + s * T;
    for (int64_t j = 0; j < T; ++j) run[j] = 0;
    for (int64_t t = 0; t < T; ++t) {
      /* update run[j] for this t: run_t[j] = q[t]==k[j] ? run_{t-1}[j-1] + 1 : 0 */
      const int qt = qs[t] > 0;
      for (int64_t j = t - 1; j >= 1; --j) run[j] = ((ks[j] > 0) == qt) ? run[j - 1] + 1 : 0;
      if (t >= 1) run[0] = ((ks[0] > 0) == qt) ? 1 : 0;
      int best = 0;
      int64_t bestj = -1;
      for (int64_t j = t - 1; j >= 0; --j) {
        int l = run[j];
        if (l > max_len) l = max_len;
        if (l > j + 1) l = (int)(j + 1);
        if (l > best) {
          best = l;
          bestj = j;
        }
      }
      sign[s * T + t] = bestj >= 0 ? (vs[bestj + 1] > 0 ? 1.f : -1.f) : -1.f;
      if (mlen) mlen[s * T + t] = best;
      if (mend) mend[s * T + t] = (int32_t)bestj;
    }
  }
}
