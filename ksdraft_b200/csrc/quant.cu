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

int ksd8_quantize_rows_launch(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t ldx,
                              int group, int flags, float dither, uint64_t seed, uint64_t offset,
                              int8_t* codes, int64_t ldc, void* scales, cudaStream_t stream) {
  QRowArgs a;
  a.x = x; a.rows = rows; a.k = k; a.ldx = ldx; a.ldc = ldc; a.group = group; a.flags = flags;
  a.dither2 = 2.0f * dither; a.seed = seed; a.offset = offset; a.codes = codes;
  a.scales = reinterpret_cast<__half*>(scales);
  const int64_t work = rows * (((k + 127) / 128 + QR_U - 1) / QR_U);
  if (work == 0) return KSD8_OK;
  const int blocks = grid_for(work, 8);
  switch (x_dtype) {
    case KSD8_F32: quantize_rows_kernel<float><<<blocks, 256, 0, stream>>>(a); break;
    case KSD8_F16: quantize_rows_kernel<__half><<<blocks, 256, 0, stream>>>(a); break;
    case KSD8_BF16: quantize_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(a); break;
    default: return KSD8_ERR_DTYPE;
  }
  return KSD8_OK;
}

int ksd8_quantize_cols_launch(const void* x, int x_dtype, const void* x_scales, int x_group,
                              int64_t rows, int64_t cols, int64_t ldx, int flags, int8_t* codes_t,
                              int64_t ldct, void* scales_t, cudaStream_t stream) {
  QColArgs a;
  a.x = x; a.x_scales = reinterpret_cast<const __half*>(x_scales); a.x_group = x_group;
  a.rows = rows; a.cols = cols; a.ldx = ldx; a.ldct = ldct; a.flags = flags;
  a.codes_t = codes_t; a.scales_t = reinterpret_cast<__half*>(scales_t);
  if (rows == 0 || cols == 0) return KSD8_OK;
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
