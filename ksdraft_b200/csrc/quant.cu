// GS128 symmetric int8 quantisers (ksdraft/kernels/quant.py:30-52 and the
// PTQR dither of ksdraft/train/stages.py:27-50).
//
// Per group of `group` consecutive elements along the quantised dimension
// (zero padded to a whole group):
//   amax  = max |x|
//   scale = fp16( clamp(amax / 127, 2^-24, 65504) )      (fp32 IEEE division)
//   code  = clamp( rint(x / scale [+ dither noise]), -127, 127 )
// The dither noise is (U - 0.5) * (2 * dither) with U from Philox4x32-10 at
// element index offset + row * Kp + col (Kp = padded row length).
//
// quantize_rows_kernel: one warp per (row, group), memory-bound, coalesced.
// quantize_cols_kernel: x^T quantised along the rows of x; a 128 x 128 tile
//   is staged in shared memory so both the reads of x (16-byte vectors) and the
//   writes of x^T are coalesced; also dequantises int8 codes on the fly
//   (dequant -> transpose -> requant of ks3_int8.py:350, :407-424).
// Codes use gs_code_fast: a reciprocal multiply with an exact fallback near
// rounding ties, bit-identical to rint(x / scale).
#include "common.cuh"

namespace ksd8 {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<int8_t>(int8_t v) { return (float)v; }

__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }

// Load 4 consecutive elements starting at column c (masked to < k).
template <typename T>
__device__ __forceinline__ void load4(const T* row, int64_t c, int64_t k, float (&v)[4]) {
  if (c + 4 <= k) {
    if constexpr (sizeof(T) == 4) {
      if ((reinterpret_cast<uintptr_t>(row + c) & 15) == 0) {
        const float4 q = *reinterpret_cast<const float4*>(row + c);
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        return;
      }
    } else {
      if ((reinterpret_cast<uintptr_t>(row + c) & 7) == 0) {
        const uint2 q = *reinterpret_cast<const uint2*>(row + c);
        const T* e = reinterpret_cast<const T*>(&q);
        v[0] = to_f32<T>(e[0]); v[1] = to_f32<T>(e[1]);
        v[2] = to_f32<T>(e[2]); v[3] = to_f32<T>(e[3]);
        return;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = (c + i < k) ? to_f32<T>(row[c + i]) : 0.f;
}

struct QRowArgs {
  const void* x;
  int64_t rows, k, ldx, ldc;
  int group;  // 128
  int flags;
  float dither2;  // 2 * dither
  uint64_t seed, offset;
  int8_t* codes;
  __half* scales;
};

// Dithered code, the reference formula rint(RN(RN(x / scale) + noise))
// clamped to +-127 (ksdraft/train/stages.py:42-48), IEEE division only near a
// rounding boundary: y = x * rcp is within 2^-14 of RN(x / scale) for |y| <
// 200 (see gs_code_fast), so t = RN(y + noise) is within 2^-13 of the
// reference's t and rounds the same unless it lies within 2^-13 of a
// half-integer.
static __device__ __noinline__ int gs_code_dither_slow(float x, float scale, float noise) {
  const float t = __fadd_rn(__fdiv_rn(x, scale), noise);
  return (int)fminf(fmaxf(rintf(t), -127.f), 127.f);
}

__device__ __forceinline__ int gs_code_dither_fast(float x, float scale, float rcp, float noise) {
  const float y = __fmul_rn(x, rcp);
  const float t = __fadd_rn(y, noise);
  const float r = rintf(t);
  if (fabsf(y) < 200.f && fabsf(__fsub_rn(t, r)) < 0.4998779296875f)
    return (int)fminf(fmaxf(r, -127.f), 127.f);
  return gs_code_dither_slow(x, scale, noise);
}

constexpr int QR_U = 1;  // groups of one row per warp iteration (occupancy keeps loads in flight)

// One warp per QR_U consecutive 128-wide groups of a row per iteration: the
// QR_U loads are in flight together and the QR_U warp reductions interleave.
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(QRowArgs a) {
  const int64_t groups = (a.k + 127) / 128;
  const int64_t kp = groups * 128;
  const int64_t ublocks = (groups + QR_U - 1) / QR_U;
  const int64_t total = a.rows * ublocks;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
       w += warps) {
    const int64_t r = w / ublocks;
    const int64_t g0 = (w - r * ublocks) * QR_U;
    const T* row = reinterpret_cast<const T*>(a.x) + r * a.ldx;
    float v[QR_U][4];
#pragma unroll
    for (int u = 0; u < QR_U; ++u) {
      const int64_t c = (g0 + u) * 128 + lane * 4;
      if (g0 + u < groups) {
        load4<T>(row, c, a.k, v[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[u][i] = 0.f;
      }
    }
    float m[QR_U];
#pragma unroll
    for (int u = 0; u < QR_U; ++u) {
      if (a.flags & KSD8_Q_ROUND_F16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[u][i] = round_f16(v[u][i]);
      }
      m[u] = fmaxf(fmaxf(fabsf(v[u][0]), fabsf(v[u][1])), fmaxf(fabsf(v[u][2]), fabsf(v[u][3])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < QR_U; ++u) m[u] = fmaxf(m[u], __shfl_xor_sync(0xffffffffu, m[u], o));
#pragma unroll
    for (int u = 0; u < QR_U; ++u) {
      const int64_t g = g0 + u;
      if (g >= groups) break;
      const int64_t c = g * 128 + lane * 4;
      __half sh;
      const float scale = gs_scale_fast(m[u], &sh);
      const float rcp = rcp_approx(scale);
      int q[4];
      if (a.flags & KSD8_Q_DITHER) {
        // one Philox block serves the 4 consecutive elements when they share it
        const uint64_t base = a.offset + (uint64_t)r * kp + c;
        float uu[4];
        if ((base & 3) == 0) {
          uint32_t ctr[4] = {(uint32_t)(base >> 2), (uint32_t)(base >> 34), 0u, 0u};
          philox4x32_10(ctr, (uint32_t)a.seed, (uint32_t)(a.seed >> 32));
#pragma unroll
          for (int i = 0; i < 4; ++i) uu[i] = (float)(ctr[i] >> 8) * 5.9604644775390625e-08f;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) uu[i] = philox_uniform(a.seed, base + i);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float noise = __fmul_rn(__fsub_rn(uu[i], 0.5f), a.dither2);
          q[i] = gs_code_dither_fast(v[u][i], scale, rcp, noise);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = gs_code_fast(v[u][i], scale, rcp);
      }
      int8_t* out = a.codes + r * a.ldc + c;
      if (c + 4 <= a.k && (reinterpret_cast<uintptr_t>(out) & 3) == 0) {
        *reinterpret_cast<char4*>(out) = make_char4((char)q[0], (char)q[1], (char)q[2], (char)q[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (c + i < a.k) out[i] = (int8_t)q[i];
      }
      if (lane == 0) a.scales[r * groups + g] = sh;
    }
  }
}

// ------------------------------------------------------------ staged row quantiser
// Contiguous rows made of whole groups (ldx == k, k % 128 == 0, 16-byte
// aligned base): the input is one run of 128-element groups.  Chunks of
// QB_GROUPS groups stream through a ring of QB_STAGES shared-memory stages by
// cp.async.bulk (one thread issues, completion counted on an mbarrier), so an
// SM keeps 100-200 KB of reads in flight without spending registers on them.
// Eight lanes share a group (16 elements each, read as 16-byte vectors l, l +
// 8, ... so that a warp's shared loads are conflict-free): 3 shuffle rounds
// and one scale per lane per 16 elements.  The arithmetic is that of
// quantize_rows_kernel; codes of a normal fp16 scale use packed f32x2 math
// (gs_code4_normal).
#ifndef KSD8_QB_GROUPS
#define KSD8_QB_GROUPS 32
#endif
#ifndef KSD8_QB_STAGES
#define KSD8_QB_STAGES 3
#endif
constexpr int QB_GROUPS = KSD8_QB_GROUPS;  // groups per chunk (a multiple of 32: 8 warps x 4)
constexpr int QB_STAGES = KSD8_QB_STAGES;

template <typename T>
struct QBulk {
  static constexpr int CHUNK = QB_GROUPS * 128 * (int)sizeof(T);
  static constexpr int SMEM = QB_STAGES * CHUNK;
};

// Four consecutive elements from shared memory as floats.
template <typename T>
__device__ __forceinline__ void lds4(const uint8_t* p, float (&v)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  } else {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&q);
    v[0] = to_f32<T>(e[0]); v[1] = to_f32<T>(e[1]);
    v[2] = to_f32<T>(e[2]); v[3] = to_f32<T>(e[3]);
  }
}

// Dithered version (ksdraft/train/stages.py:42-48): noise = RN((U - 0.5) * d2)
// computed as one fma(U, d2, -d2 / 2) (U - 0.5 is exact, so the single rounding
// is the same); t = RN(y + noise) is clamped to +-127 before the shifter
// (rint and the clamp commute at the integers +-127), and a t within 2^-13 of
// a half-integer sends the four to gs_code_dither_fast.
__device__ __forceinline__ uint32_t gs_code4_dither_normal(const float (&v)[4], const float (&u)[4],
                                                           float d2, float scale, float rcp) {
  const float2 rc = make_float2(rcp, rcp), dd = make_float2(d2, d2);
  const float2 hd = make_float2(-0.5f * d2, -0.5f * d2);
  const float2 mg = make_float2(12582912.f, 12582912.f), nmg = make_float2(-12582912.f, -12582912.f);
  const float2 n01 = __ffma2_rn(make_float2(u[0], u[1]), dd, hd);
  const float2 n23 = __ffma2_rn(make_float2(u[2], u[3]), dd, hd);
  float2 t01 = __fadd2_rn(__fmul2_rn(make_float2(v[0], v[1]), rc), n01);
  float2 t23 = __fadd2_rn(__fmul2_rn(make_float2(v[2], v[3]), rc), n23);
  t01 = make_float2(fminf(fmaxf(t01.x, -127.f), 127.f), fminf(fmaxf(t01.y, -127.f), 127.f));
  t23 = make_float2(fminf(fmaxf(t23.x, -127.f), 127.f), fminf(fmaxf(t23.y, -127.f), 127.f));
  const float2 s01 = __fadd2_rn(t01, mg), s23 = __fadd2_rn(t23, mg);
  const float2 d01 = __ffma2_rn(t01, make_float2(-1.f, -1.f), __fadd2_rn(s01, nmg));
  const float2 d23 = __ffma2_rn(t23, make_float2(-1.f, -1.f), __fadd2_rn(s23, nmg));
  const float dm =
      fmax_nan(fmax_nan(fabsf(d01.x), fabsf(d01.y)), fmax_nan(fabsf(d23.x), fabsf(d23.y)));
  if (!(dm < 0.4998779296875f)) {
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float noise = __fmul_rn(__fsub_rn(u[e], 0.5f), d2);
      w |= ((uint32_t)gs_code_dither_fast(v[e], scale, rcp, noise) & 0xFFu) << (8 * e);
    }
    return w;
  }
  return __byte_perm(__byte_perm(__float_as_uint(s01.x), __float_as_uint(s01.y), 0x0040),
                     __byte_perm(__float_as_uint(s23.x), __float_as_uint(s23.y), 0x0040), 0x5410);
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_bulk_kernel(QRowArgs a, int* status) {
  extern __shared__ __align__(128) uint8_t qb_sm[];
  __shared__ __align__(8) uint64_t full[QB_STAGES];
  __shared__ int abort_s;
  volatile int* abort_flag = &abort_s;
  constexpr int CH = QBulk<T>::CHUNK;
  constexpr int VN = 16 / (int)sizeof(T);  // elements per 16-byte vector
  constexpr int NV = 16 / VN;              // vectors per lane per group (16 elements)
  constexpr int NP = QB_GROUPS / 32;       // passes of 32 groups per chunk
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int l8 = lane & 7;                 // lane within its group's 8 lanes
  // 32-bit group indexing: the launcher sends only rows * k / 128 < 2^31 here
  const uint32_t gpr = (uint32_t)(a.k >> 7);  // groups per row
  const uint32_t ng = (uint32_t)(a.rows * (int64_t)gpr);
  const uint32_t nch = (ng + QB_GROUPS - 1) / QB_GROUPS;
  const int my_n = blockIdx.x < nch ? (int)((nch - 1 - blockIdx.x) / gridDim.x + 1) : 0;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(a.x);

  auto issue = [&](int i) {  // this CTA's i-th chunk into stage i % QB_STAGES
    const uint32_t g0 = (blockIdx.x + (uint32_t)i * gridDim.x) * QB_GROUPS;
    const uint32_t n = ng - g0 < QB_GROUPS ? ng - g0 : QB_GROUPS;
    const uint32_t bytes = n * 128u * (uint32_t)sizeof(T);
    uint64_t* bar = &full[i % QB_STAGES];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load_g2s(qb_sm + (i % QB_STAGES) * CH, src + (uint64_t)g0 * 128 * sizeof(T), bytes, bar);
  };
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < QB_STAGES; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    for (int i = 0; i < QB_STAGES && i < my_n; ++i) issue(i);
  }
  // (row, group) of this thread's group in each pass, tracked without a
  // division per chunk: chunk i of this CTA starts step * i groups after chunk 0.
  uint32_t off_r[NP], off_g[NP];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const uint32_t off = p * 32 + warp * 4 + (lane >> 3);
    off_r[p] = off / gpr;
    off_g[p] = off - off_r[p] * gpr;
  }
  const uint32_t step = gridDim.x * QB_GROUPS;
  const uint32_t step_r = step / gpr, step_g = step - step_r * gpr;
  uint32_t base_r = blockIdx.x * QB_GROUPS / gpr;
  uint32_t base_g = blockIdx.x * QB_GROUPS - base_r * gpr;
  __syncthreads();

  const bool rf16 = (a.flags & KSD8_Q_ROUND_F16) != 0, dither = (a.flags & KSD8_Q_DITHER) != 0;
  int consumed = 0, issued = my_n < QB_STAGES ? my_n : QB_STAGES;
  for (int i = 0; i < my_n; ++i) {
    const bool got =
        q_wait(&full[i % QB_STAGES], (uint32_t)((i / QB_STAGES) & 1), abort_flag, status);
    if (!__syncthreads_and(got && !*abort_flag)) break;  // every thread leaves together
    consumed = i + 1;
    // every thread is past chunk i - 1: its stage takes chunk i - 1 + QB_STAGES
    if (i >= 1 && i - 1 + QB_STAGES < my_n) {
      if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        issue(i - 1 + QB_STAGES);
      }
      issued = i + QB_STAGES;
    }
    const uint32_t chunk_g0 = (blockIdx.x + (uint32_t)i * gridDim.x) * QB_GROUPS;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      // 8 lanes per group, 4 groups per warp: lane l8 holds the 16-byte vectors
      // l8, l8 + 8, ... of its group (consecutive lanes, consecutive vectors)
      const int gq = p * 32 + warp * 4 + (lane >> 3);  // group within the chunk
      const uint8_t* gsm = qb_sm + (i % QB_STAGES) * CH + gq * 128 * (int)sizeof(T);
      float v[NV][VN];
      float mx = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) {  // a group past the end reads stale bytes, never stored
        const uint4 raw = *reinterpret_cast<const uint4*>(gsm + (l8 + 8 * k) * 16);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          float x = to_f32<T>(e[j]);
          if (rf16) x = round_f16(x);
          v[k][j] = x;
          mx = fmaxf(mx, fabsf(x));
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      uint32_t r = base_r + off_r[p], g = base_g + off_g[p];
      if (g >= gpr) {
        g -= gpr;
        ++r;
      }
      if (chunk_g0 + gq >= ng) continue;
      __half sh;
      const float scale = gs_scale_fast(mx, &sh);
      const float rcp = rcp_approx(scale);
      const bool normal = !(mx > 0.f && (!(scale >= 6.103515625e-05f) || !(mx <= 8.0e6f)));
      uint32_t w[NV][VN / 4];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const uint32_t c = g * 128 + (l8 + 8 * k) * VN;  // column of the vector's first element
#pragma unroll
        for (int q = 0; q < VN / 4; ++q) {
          const float* x4 = &v[k][4 * q];
          uint32_t word = 0;
          if (dither) {
            const uint64_t base = a.offset + (uint64_t)r * (uint64_t)a.k + c + 4 * q;
            float uu[4];
            if ((base & 3) == 0) {
              uint32_t ctr[4] = {(uint32_t)(base >> 2), (uint32_t)(base >> 34), 0u, 0u};
              philox4x32_10(ctr, (uint32_t)a.seed, (uint32_t)(a.seed >> 32));
#pragma unroll
              for (int e = 0; e < 4; ++e) uu[e] = (float)(ctr[e] >> 8) * 5.9604644775390625e-08f;
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) uu[e] = philox_uniform(a.seed, base + e);
            }
            if (normal && a.dither2 <= 1024.f) {
              const float xv[4] = {x4[0], x4[1], x4[2], x4[3]};
              word = gs_code4_dither_normal(xv, uu, a.dither2, scale, rcp);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float noise = __fmul_rn(__fsub_rn(uu[e], 0.5f), a.dither2);
                word |= ((uint32_t)gs_code_dither_fast(x4[e], scale, rcp, noise) & 0xFFu)
                        << (8 * e);
              }
            }
          } else if (!normal) {  // subnormal or clamped scale: per-element path with saturation
#pragma unroll
            for (int e = 0; e < 4; ++e)
              word |= ((uint32_t)gs_code_fast(x4[e], scale, rcp) & 0xFFu) << (8 * e);
          } else {
            const float xv[4] = {x4[0], x4[1], x4[2], x4[3]};
            word = gs_code4_normal(xv, scale, rcp);
          }
          w[k][q] = word;
        }
        int8_t* out = a.codes + (uint64_t)r * a.ldc + c;
        if constexpr (VN == 4) {
          *reinterpret_cast<uint32_t*>(out) = w[k][0];
        } else {
          *reinterpret_cast<uint2*>(out) = make_uint2(w[k][0], w[k][1]);
        }
      }
      if (l8 == 0) a.scales[(uint64_t)r * gpr + g] = sh;
    }
    base_r += step_r;
    base_g += step_g;
    if (base_g >= gpr) {
      base_g -= gpr;
      ++base_r;
    }
  }
  // After a timeout: let the copies still in flight land (bounded) before the
  // CTA's shared memory is released.
  if (threadIdx.x == 0 && *abort_flag) {
    for (int i = consumed; i < issued; ++i) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[i % QB_STAGES], (uint32_t)((i / QB_STAGES) & 1)) &&
             globaltimer_ns() - t0 < KSD8_WAIT_NS) {
      }
    }
  }
}

struct QColArgs {
  const void* x;
  const __half* x_scales;
  int x_group;
  int64_t rows, cols, ldx, ldct;
  int flags;
  int8_t* codes_t;
  __half* scales_t;
};

constexpr int QC_TR = 128;  // rows per tile (one output group along the rows)
constexpr int QC_TC = 128;  // columns per tile

template <typename T>
struct QColTile {
  static constexpr int ROW_BYTES = QC_TC * (int)sizeof(T) + 16;  // padded source row
  static constexpr int SMEM = QC_TR * ROW_BYTES + QC_TR * 4;     // + per-row dequant scale
};

template <typename T>
__device__ __forceinline__ float qcol_val(const uint8_t* tile, int rr, int cc) {
  return to_f32<T>(*reinterpret_cast<const T*>(tile + rr * QColTile<T>::ROW_BYTES +
                                               cc * (int)sizeof(T)));
}

// One CTA per 128 x 128 tile.  The tile is staged in shared memory in its
// source type (int8 codes: 18 KB, so up to 8 CTAs per SM keep loads in
// flight) by coalesced 16-byte row loads; int8 codes keep one dequantisation
// scale per row (with GS128 input scales a 128-column tile lies in one input
// group), applied when the values are read back.
template <typename T, bool DEQUANT>
__global__ void __launch_bounds__(256) quantize_cols_kernel(QColArgs a) {
  extern __shared__ __align__(16) uint8_t qsm[];
  using TL = QColTile<T>;
  float* rscale = reinterpret_cast<float*>(qsm + QC_TR * TL::ROW_BYTES);
  const int64_t r0 = (int64_t)blockIdx.y * QC_TR;
  const int64_t c0 = (int64_t)blockIdx.x * QC_TC;
  const int tid = threadIdx.x;
  constexpr int VN = 16 / (int)sizeof(T);   // elements per 16-byte vector
  constexpr int VPR = QC_TC / VN;           // vectors per tile row
  const int64_t xs_groups = DEQUANT ? (a.cols + a.x_group - 1) / a.x_group : 0;
  const bool vec_ok = (a.ldx * (int64_t)sizeof(T)) % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && c0 + QC_TC <= a.cols;
  if constexpr (DEQUANT) {
    for (int rr = tid; rr < QC_TR; rr += 256) {
      const int64_t r = r0 + rr;
      rscale[rr] = r < a.rows ? __half2float(a.x_scales[r * xs_groups + c0 / a.x_group]) : 0.f;
    }
  }
  for (int idx = tid; idx < QC_TR * VPR; idx += 256) {
    const int rr = idx / VPR, vv = idx % VPR;
    const int64_t r = r0 + rr;
    const int64_t c = c0 + vv * VN;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (r < a.rows) {
      const T* row = reinterpret_cast<const T*>(a.x) + r * a.ldx;
      if (vec_ok) {
        raw = __ldcs(reinterpret_cast<const uint4*>(row + c));
      } else {
        T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int i = 0; i < VN; ++i) e[i] = (c + i < a.cols) ? row[c + i] : T(0);
      }
    }
    *reinterpret_cast<uint4*>(qsm + rr * TL::ROW_BYTES + vv * 16) = raw;
  }
  // Column phase: thread t owns column t % 128 and rows (t / 128) * 64 .. +64:
  // per-thread amax (consecutive lanes read consecutive columns), one
  // exchange for the other half, and 64 codes written as 16-byte vectors of
  // the x^T row.
  __shared__ float s_amax[2][QC_TC];
  __syncthreads();
  const int cc = tid & (QC_TC - 1), half = tid >> 7;
  const int64_t c = c0 + cc;
  const bool rf16 = !DEQUANT && (a.flags & KSD8_Q_ROUND_F16);
  auto val = [&](int rr) -> float {
    float v = qcol_val<T>(qsm, rr, cc);
    if constexpr (DEQUANT) v = v * rscale[rr];
    else if (rf16) v = round_f16(v);
    return v;
  };
  float m = 0.f;
#pragma unroll 16
  for (int i = 0; i < 64; ++i) m = fmaxf(m, fabsf(val(half * 64 + i)));
  s_amax[half][cc] = m;
  __syncthreads();
  if (c >= a.cols) return;
  m = fmaxf(s_amax[0][cc], s_amax[1][cc]);
  const int64_t rgroups = (a.rows + 127) / 128;
  __half sh;
  const float scale = gs_scale_fast(m, &sh);
  const float rcp = rcp_approx(scale);
  const int64_t rb = r0 + half * 64;
  int8_t* out = a.codes_t + c * a.ldct + rb;
  if (rb + 64 <= a.rows && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int q = gs_code_fast(val(half * 64 + v * 16 + j * 4 + b), scale, rcp);
          word |= (uint32_t)(q & 0xFF) << (8 * b);
        }
        w[j] = word;
      }
      *reinterpret_cast<uint4*>(out + v * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    for (int i = 0; i < 64; ++i)
      if (rb + i < a.rows) out[i] = (int8_t)gs_code_fast(val(half * 64 + i), scale, rcp);
  }
  if (half == 0) a.scales_t[c * rgroups + blockIdx.y] = sh;
}

// ------------------------------------------------------------ TMA-staged transposed quantiser
// x^T quantised along the rows of x, 128 x 128 tiles of x brought in by 2D
// TMA loads (zero fill past the edges, which is the reference's group
// padding) through a ring of QTma<T>::STAGES stages; persistent CTAs take
// tiles blockIdx.x, + gridDim.x, ...  Thread layout per tile: warp w owns
// rows 16w .. 16w+15, lane l owns columns 4l .. 4l+3 (conflict-free 4/8/16-byte
// shared loads along a row); the column amax is combined across the 8 warps
// through shared memory (the one CTA barrier per tile), and each thread
// writes its 4 columns' 16 codes as one 16-byte vector per column of x^T.
// Codes: y = v * RN(1/scale) rounded with the 1.5 * 2^23 shifter on packed
// f32x2 arithmetic.  For a normal fp16 scale below the upper clamp |y| <=
// 127.07, so the shifter's low byte is the code, saturation never applies,
// and rint(y) equals rint(RN(v / scale)) unless y lies within 2^-13 of a
// half-integer: a row of 4 codes holding such a value is recomputed with the
// IEEE division (out of line, taken for ~0.1% of the rows), and a thread with a
// non-zero column outside that scale range recomputes all of its 64 codes.
constexpr int QT_R = 128, QT_C = 128;

#ifndef KSD8_QT_STAGES_I8
#define KSD8_QT_STAGES_I8 2
#endif
#ifndef KSD8_QT_MIN_CTAS_I8
#define KSD8_QT_MIN_CTAS_I8 4
#endif
template <typename T>
struct QTma {
  static constexpr int TILE = QT_R * QT_C * (int)sizeof(T);
  static constexpr int STAGES = sizeof(T) == 1 ? KSD8_QT_STAGES_I8 : (sizeof(T) == 2 ? 3 : 2);
  static constexpr int SMEM = STAGES * TILE + 1024;  // + slack for 1024-byte alignment
  static constexpr int MIN_CTAS = sizeof(T) == 1 ? KSD8_QT_MIN_CTAS_I8 : (sizeof(T) == 2 ? 2 : 1);
};

// Columns 4l .. 4l+3 of one tile row as floats.  int8 codes are dequantised
// exactly: byte b ^ 0x80 placed under the exponent of 2^23 gives 2^23 + code +
// 128, and (that - (2^23 + 128)) * rs is code * rs (a product of at most 19
// significant bits, exact in fp32).
template <typename T, bool DEQUANT>
__device__ __forceinline__ void qt_row4(const uint8_t* p, float rs, bool rf16, float2& v01,
                                        float2& v23) {
  if constexpr (DEQUANT) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p) ^ 0x80808080u;
    const float2 bias = make_float2(-8388736.f, -8388736.f);
    const float2 rs2 = make_float2(rs, rs);
    const float2 f01 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650)),
                                   __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7651)));
    const float2 f23 = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7652)),
                                   __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7653)));
    v01 = __fmul2_rn(__fadd2_rn(f01, bias), rs2);
    v23 = __fmul2_rn(__fadd2_rn(f23, bias), rs2);
  } else {
    if constexpr (sizeof(T) == 4) {
      const float4 q = *reinterpret_cast<const float4*>(p);
      v01 = make_float2(q.x, q.y);
      v23 = make_float2(q.z, q.w);
    } else {
      const uint2 q = *reinterpret_cast<const uint2*>(p);
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        v01 = make_float2(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u));
        v23 = make_float2(__uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u));
      } else {
        v01 = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
        v23 = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
      }
    }
    if (rf16) {
      v01 = __half22float2(__float22half2_rn(v01));
      v23 = __half22float2(__float22half2_rn(v23));
    }
  }
}

// The 4 codes of one tile row (columns 4l .. 4l+3) by IEEE division, byte j =
// column j.  Out of line: taken only next to rounding ties.
template <typename T, bool DEQUANT>
static __device__ __noinline__ uint32_t qt_exact_row(const uint8_t* row, float rs, bool rf16,
                                                     float s0, float s1, float s2, float s3) {
  float2 v01, v23;
  qt_row4<T, DEQUANT>(row, rs, rf16, v01, v23);
  return ((uint32_t)gs_code(v01.x, s0) & 0xFFu) | (((uint32_t)gs_code(v01.y, s1) & 0xFFu) << 8) |
         (((uint32_t)gs_code(v23.x, s2) & 0xFFu) << 16) |
         (((uint32_t)gs_code(v23.y, s3) & 0xFFu) << 24);
}

// The 64 codes of one thread (4 columns x 16 rows) by IEEE division, packed
// as in the fast path: out[4 * column + row / 4], row % 4 in byte order.
// Out of line, so that the fast path keeps its registers.
template <typename T, bool DEQUANT>
static __device__ __noinline__ void qt_exact_codes(const uint8_t* rows16, const float* rsw,
                                                   bool rf16, float s0, float s1, float s2,
                                                   float s3, uint32_t* out) {
  const float sc[4] = {s0, s1, s2, s3};
  for (int i = 0; i < 16; ++i) out[i] = 0u;
  for (int rr = 0; rr < 16; ++rr) {
    float2 v01, v23;
    qt_row4<T, DEQUANT>(rows16 + rr * QT_C * (int)sizeof(T), DEQUANT ? rsw[rr] : 0.f, rf16, v01,
                        v23);
    const float v[4] = {v01.x, v01.y, v23.x, v23.y};
    for (int j = 0; j < 4; ++j)
      out[j * 4 + (rr >> 2)] |= ((uint32_t)gs_code(v[j], sc[j]) & 0xFFu) << ((rr & 3) * 8);
  }
}

template <typename T, bool DEQUANT>
__global__ void __launch_bounds__(256, QTma<T>::MIN_CTAS)
    quantize_cols_tma_kernel(const __grid_constant__ CUtensorMap tm, QColArgs a, int* status) {
  constexpr int S = QTma<T>::STAGES, TB = QTma<T>::TILE, ES = (int)sizeof(T);
  extern __shared__ uint8_t qt_raw[];
  uint8_t* qt = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qt_raw) + 1023) &
                                           ~uintptr_t(1023));
  __shared__ __align__(16) float s_amax[2][8][QT_C];
  __shared__ __align__(16) float s_rs[2][QT_R];
  __shared__ __align__(8) uint64_t full[S];
  __shared__ int abort_s;
  volatile int* abort_flag = &abort_s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // 32-bit tile indexing: rows, cols < 2^31, so fewer than 2^31 tiles
  const uint32_t nx = (uint32_t)((a.cols + QT_C - 1) / QT_C);
  const uint32_t ny = (uint32_t)((a.rows + QT_R - 1) / QT_R);
  const uint32_t ntiles = nx * ny;
  const int my_n = blockIdx.x < ntiles ? (int)((ntiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;
  const int64_t xs_groups = DEQUANT ? (a.cols + a.x_group - 1) / a.x_group : 0;
  const uint32_t tiles_per_xgroup = DEQUANT ? (uint32_t)(a.x_group / QT_C) : 1u;
  const bool rf16 = !DEQUANT && (a.flags & KSD8_Q_ROUND_F16);

  auto issue = [&](int i) {  // this CTA's i-th tile into stage i % S
    const uint32_t t = blockIdx.x + (uint32_t)i * gridDim.x;
    const uint32_t ty = t / nx, tx = t - ty * nx;
    uint64_t* bar = &full[i % S];
    mbar_arrive_expect_tx(bar, TB);
    tma_load_2d(qt + (i % S) * TB, &tm, bar, (int32_t)(tx * QT_C), (int32_t)(ty * QT_R));
  };
  // Dequantisation scale of row 16 * warp + lane (lanes 0..15) of tile i,
  // loaded one tile ahead of its use.
  auto load_rs = [&](int i) -> float {
    if (!DEQUANT || lane >= 16 || i >= my_n) return 0.f;
    const uint32_t t = blockIdx.x + (uint32_t)i * gridDim.x;
    const uint32_t ty = t / nx, tx = t - ty * nx;
    const int64_t r = (int64_t)ty * QT_R + warp * 16 + lane;
    return r < a.rows ? __half2float(a.x_scales[r * xs_groups + tx / tiles_per_xgroup]) : 0.f;
  };
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm);
    for (int i = 0; i < S && i < my_n; ++i) issue(i);
  }
  float rs_next = load_rs(0);
  __syncthreads();

  const float2 magic2 = make_float2(12582912.f, 12582912.f);
  const float2 nmagic2 = make_float2(-12582912.f, -12582912.f);
  const float2 neg1 = make_float2(-1.f, -1.f);
  int consumed = 0, issued = my_n < S ? my_n : S;
  for (int i = 0; i < my_n; ++i) {
    const int b = i & 1;
    if constexpr (DEQUANT) {
      if (lane < 16) s_rs[b][warp * 16 + lane] = rs_next;
      rs_next = load_rs(i + 1);
      __syncwarp();
    }
    const bool got = q_wait(&full[i % S], (uint32_t)((i / S) & 1), abort_flag, status);
    const uint8_t* rows16 = qt + (i % S) * TB + (warp * 16 * QT_C + lane * 4) * ES;
    const float* rsw = &s_rs[b][warp * 16];

    // pass 1: amax of each of the 4 columns over this warp's 16 rows
    float m[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) {
      float2 v01, v23;
      qt_row4<T, DEQUANT>(rows16 + rr * QT_C * ES, DEQUANT ? rsw[rr] : 0.f, rf16, v01, v23);
      m[0] = fmaxf(m[0], fabsf(v01.x));
      m[1] = fmaxf(m[1], fabsf(v01.y));
      m[2] = fmaxf(m[2], fabsf(v23.x));
      m[3] = fmaxf(m[3], fabsf(v23.y));
    }
    *reinterpret_cast<float4*>(&s_amax[b][warp][lane * 4]) = make_float4(m[0], m[1], m[2], m[3]);
    if (!__syncthreads_and(got && !*abort_flag)) break;  // every thread leaves together
    consumed = i + 1;
    // every thread is past tile i - 1: its stage takes tile i - 1 + S
    if (i >= 1 && i - 1 + S < my_n) {
      if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        issue(i - 1 + S);
      }
      issued = i + S;
    }
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float4 p = *reinterpret_cast<const float4*>(&s_amax[b][w][lane * 4]);
      m[0] = fmaxf(m[0], p.x);
      m[1] = fmaxf(m[1], p.y);
      m[2] = fmaxf(m[2], p.z);
      m[3] = fmaxf(m[3], p.w);
    }
    __half sh[4];
    float sc[4], rc[4];
    bool exact = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sc[j] = gs_scale_fast(m[j], &sh[j]);
      rc[j] = rcp_approx(sc[j]);
      exact |= m[j] > 0.f && (!(sc[j] >= 6.103515625e-05f) || !(m[j] <= 8.0e6f));
    }
    const float2 rc01 = make_float2(rc[0], rc[1]), rc23 = make_float2(rc[2], rc[3]);

    // pass 2: codes, four rows at a time packed into one word per column
    uint32_t words[4][4];  // [column][row quad]
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t tb[4][4];  // [row][column]: shifter words, code in the low byte
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int rr = k * 4 + q;
        float2 v01, v23;
        qt_row4<T, DEQUANT>(rows16 + rr * QT_C * ES, DEQUANT ? rsw[rr] : 0.f, rf16, v01, v23);
        const float2 y01 = __fmul2_rn(v01, rc01), y23 = __fmul2_rn(v23, rc23);
        const float2 t01 = __fadd2_rn(y01, magic2), t23 = __fadd2_rn(y23, magic2);
        const float2 d01 = __ffma2_rn(y01, neg1, __fadd2_rn(t01, nmagic2));
        const float2 d23 = __ffma2_rn(y23, neg1, __fadd2_rn(t23, nmagic2));
        tb[q][0] = __float_as_uint(t01.x);
        tb[q][1] = __float_as_uint(t01.y);
        tb[q][2] = __float_as_uint(t23.x);
        tb[q][3] = __float_as_uint(t23.y);
        const float dm =
            fmax_nan(fmax_nan(fabsf(d01.x), fabsf(d01.y)), fmax_nan(fabsf(d23.x), fabsf(d23.y)));
        if (!(dm < 0.4998779296875f)) {  // near a rounding tie: IEEE division for this row
          const uint32_t fix = qt_exact_row<T, DEQUANT>(
              rows16 + rr * QT_C * ES, DEQUANT ? rsw[rr] : 0.f, rf16, sc[0], sc[1], sc[2], sc[3]);
#pragma unroll
          for (int j = 0; j < 4; ++j) tb[q][j] = (fix >> (8 * j)) & 0xFFu;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        words[j][k] = __byte_perm(__byte_perm(tb[0][j], tb[1][j], 0x0040),
                                  __byte_perm(tb[2][j], tb[3][j], 0x0040), 0x5410);
    }
    if (exact) {  // rare: IEEE division for all 64 codes
      uint32_t ex[16];
      qt_exact_codes<T, DEQUANT>(rows16, rsw, rf16, sc[0], sc[1], sc[2], sc[3], ex);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int k = 0; k < 4; ++k) words[j][k] = ex[j * 4 + k];
    }

    const uint32_t t = blockIdx.x + (uint32_t)i * gridDim.x;
    const uint32_t ty = t / nx, tx = t - ty * nx;
    const int64_t r0 = (int64_t)ty * QT_R + warp * 16;
    const int64_t cb = (int64_t)tx * QT_C + lane * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = cb + j;
      if (c >= a.cols) break;
      int8_t* out = a.codes_t + c * a.ldct + r0;
      if (r0 + 16 <= a.rows && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        *reinterpret_cast<uint4*>(out) =
            make_uint4(words[j][0], words[j][1], words[j][2], words[j][3]);
      } else {
        for (int e = 0; e < 16 && r0 + e < a.rows; ++e)
          out[e] = (int8_t)((words[j][e >> 2] >> ((e & 3) * 8)) & 0xFFu);
      }
      if (warp == 0) a.scales_t[c * ny + ty] = sh[j];
    }
  }
  // After a timeout: let the copies still in flight land (bounded) before the
  // CTA's shared memory is released.
  if (threadIdx.x == 0 && *abort_flag) {
    for (int i = consumed; i < issued; ++i) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[i % S], (uint32_t)((i / S) & 1)) &&
             globaltimer_ns() - t0 < KSD8_WAIT_NS) {
      }
    }
  }
}

__global__ void philox_uniform_kernel(uint64_t seed, uint64_t offset, int64_t n, float* out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = philox_uniform(seed, offset + i);
}

}  // namespace ksd8

using namespace ksd8;

static int grid_for(int64_t work_items, int per_block, int max_blocks = 148 * 16) {
  int64_t b = (work_items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return (int)b;
}

// CTAs per SM for a kernel with `smem` bytes of dynamic shared memory (228 KB
// per SM, 1 KB reserved per CTA, at most 8 CTAs of 256 threads).
static int ctas_per_sm(int smem) {
  const int n = (228 * 1024) / (smem + 1024 + 64);
  return n < 1 ? 1 : (n > 8 ? 8 : n);
}

template <typename T>
static int launch_rows_bulk(const QRowArgs& a, int* status, cudaStream_t stream) {
  static unsigned attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 32) return KSD8_ERR_UNSUPPORTED;
  if (!(attr_dev_mask & (1u << dev))) {
    if (cudaFuncSetAttribute(quantize_rows_bulk_kernel<T>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             QBulk<T>::SMEM) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    attr_dev_mask |= (1u << dev);
  }
  const int64_t chunks = (a.rows * (a.k / 128) + QB_GROUPS - 1) / QB_GROUPS;
  const int64_t cap = (int64_t)current_sm_count() * ctas_per_sm(QBulk<T>::SMEM);
  const unsigned grid = (unsigned)(chunks < cap ? chunks : cap);
  quantize_rows_bulk_kernel<T><<<grid, 256, QBulk<T>::SMEM, stream>>>(a, status);
  return KSD8_OK;
}

int ksd8_quantize_rows_launch(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t ldx,
                              int group, int flags, float dither, uint64_t seed, uint64_t offset,
                              int8_t* codes, int64_t ldc, void* scales, int* status,
                              cudaStream_t stream) {
  QRowArgs a;
  a.x = x; a.rows = rows; a.k = k; a.ldx = ldx; a.ldc = ldc; a.group = group; a.flags = flags;
  a.dither2 = 2.0f * dither; a.seed = seed; a.offset = offset; a.codes = codes;
  a.scales = reinterpret_cast<__half*>(scales);
  const int64_t work = rows * (((k + 127) / 128 + QR_U - 1) / QR_U);
  if (work == 0) return KSD8_OK;
  // Staged kernel: one contiguous run of whole groups, 16-byte aligned source,
  // 4-byte aligned code rows.
  const bool staged = !(flags & KSD8_Q_PLAIN_LOADS) && ldx == k && (k % 128) == 0 &&
                      rows * (k / 128) < (int64_t(1) << 31) &&
                      (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(codes) & 3) == 0 && (ldc % 4) == 0;
  if (staged) {
    switch (x_dtype) {
      case KSD8_F32: return launch_rows_bulk<float>(a, status, stream);
      case KSD8_F16: return launch_rows_bulk<__half>(a, status, stream);
      case KSD8_BF16: return launch_rows_bulk<__nv_bfloat16>(a, status, stream);
      default: return KSD8_ERR_DTYPE;
    }
  }
  const int blocks = grid_for(work, 8);
  switch (x_dtype) {
    case KSD8_F32: quantize_rows_kernel<float><<<blocks, 256, 0, stream>>>(a); break;
    case KSD8_F16: quantize_rows_kernel<__half><<<blocks, 256, 0, stream>>>(a); break;
    case KSD8_BF16: quantize_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(a); break;
    default: return KSD8_ERR_DTYPE;
  }
  return KSD8_OK;
}

// x (rows, cols) with row stride ld elements as 128 x 128 boxes, no swizzle,
// zero fill outside.  False when the driver rejects the layout (then the
// thread-load kernel runs).
static bool make_tmap_tile128(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt,
                              int esize, int64_t rows, int64_t cols, int64_t ld) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)QT_C, (cuuint32_t)QT_R};
  cuuint32_t estr[2] = {1u, 1u};
  return enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <typename T, bool DEQUANT>
static int launch_cols_tma(const CUtensorMap& tm, const QColArgs& a, int* status,
                           cudaStream_t stream) {
  static unsigned attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 32) return KSD8_ERR_UNSUPPORTED;
  if (!(attr_dev_mask & (1u << dev))) {
    if (cudaFuncSetAttribute(quantize_cols_tma_kernel<T, DEQUANT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             QTma<T>::SMEM) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    attr_dev_mask |= (1u << dev);
  }
  const int64_t tiles = ((a.rows + QT_R - 1) / QT_R) * ((a.cols + QT_C - 1) / QT_C);
  const int64_t cap = (int64_t)current_sm_count() * QTma<T>::MIN_CTAS;
  const unsigned grid = (unsigned)(tiles < cap ? tiles : cap);
  quantize_cols_tma_kernel<T, DEQUANT><<<grid, 256, QTma<T>::SMEM, stream>>>(tm, a, status);
  return KSD8_OK;
}

int ksd8_quantize_cols_launch(const void* x, int x_dtype, const void* x_scales, int x_group,
                              int64_t rows, int64_t cols, int64_t ldx, int flags, int8_t* codes_t,
                              int64_t ldct, void* scales_t, int* status, cudaStream_t stream) {
  QColArgs a;
  a.x = x; a.x_scales = reinterpret_cast<const __half*>(x_scales); a.x_group = x_group;
  a.rows = rows; a.cols = cols; a.ldx = ldx; a.ldct = ldct; a.flags = flags;
  a.codes_t = codes_t; a.scales_t = reinterpret_cast<__half*>(scales_t);
  if (rows == 0 || cols == 0) return KSD8_OK;
  {
    int esize = 0;
    CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    switch (x_dtype) {
      case KSD8_F32: esize = 4; dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
      case KSD8_F16: esize = 2; dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
      case KSD8_BF16: esize = 2; dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
      case KSD8_I8: esize = 1; dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
      default: return KSD8_ERR_DTYPE;
    }
    CUtensorMap tm;
    const bool staged = !(flags & KSD8_Q_PLAIN_LOADS) &&
                        (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx * esize) % 16 == 0 &&
                        rows < (int64_t(1) << 31) && cols < (int64_t(1) << 31) &&
                        make_tmap_tile128(&tm, x, dt, esize, rows, cols, ldx);
    if (staged) {
      switch (x_dtype) {
        case KSD8_F32: return launch_cols_tma<float, false>(tm, a, status, stream);
        case KSD8_F16: return launch_cols_tma<__half, false>(tm, a, status, stream);
        case KSD8_BF16: return launch_cols_tma<__nv_bfloat16, false>(tm, a, status, stream);
        default: return launch_cols_tma<int8_t, true>(tm, a, status, stream);
      }
    }
  }
  dim3 grid((unsigned)((cols + QC_TC - 1) / QC_TC), (unsigned)((rows + QC_TR - 1) / QC_TR));
  static unsigned attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1u << dev))) {
    cudaFuncSetAttribute(quantize_cols_kernel<float, false>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, QColTile<float>::SMEM);
    cudaFuncSetAttribute(quantize_cols_kernel<__half, false>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, QColTile<__half>::SMEM);
    cudaFuncSetAttribute(quantize_cols_kernel<__nv_bfloat16, false>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         QColTile<__nv_bfloat16>::SMEM);
    cudaFuncSetAttribute(quantize_cols_kernel<int8_t, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, QColTile<int8_t>::SMEM);
    attr_dev_mask |= (1u << dev);
  }
  switch (x_dtype) {
    case KSD8_F32:
      quantize_cols_kernel<float, false><<<grid, 256, QColTile<float>::SMEM, stream>>>(a);
      break;
    case KSD8_F16:
      quantize_cols_kernel<__half, false><<<grid, 256, QColTile<__half>::SMEM, stream>>>(a);
      break;
    case KSD8_BF16:
      quantize_cols_kernel<__nv_bfloat16, false>
          <<<grid, 256, QColTile<__nv_bfloat16>::SMEM, stream>>>(a);
      break;
    case KSD8_I8:
      quantize_cols_kernel<int8_t, true><<<grid, 256, QColTile<int8_t>::SMEM, stream>>>(a);
      break;
    default: return KSD8_ERR_DTYPE;
  }
  return KSD8_OK;
}

int ksd8_philox_launch(uint64_t seed, uint64_t offset, int64_t n, float* out, cudaStream_t stream) {
  if (n == 0) return KSD8_OK;
  philox_uniform_kernel<<<grid_for(n, 256), 256, 0, stream>>>(seed, offset, n, out);
  return KSD8_OK;
}
