// LM head (vocab projection) kernels around the W8A8 GEMM: vocab-parallel
// cross-entropy partials and gradient, and per-row top-k for drafting.
//
// The reference head is a tied fp32 nn.Linear(d, V) followed by
// F.cross_entropy (ksdraft/model/draft.py:39,51,82; ksdraft/train/__init__.py:77).
// Here each rank owns a contiguous vocab shard of the logits (M, V_local) and
// reduces it to three floats per row: the shard max, the shard sum of
// exp(logit - max) and the target logit when the target falls in the shard.
// The host combines ranks with all-reduces of those (M) vectors
// (max, then rescaled sum, then target), so no logits cross NVLink.
//
//   ce_partials_kernel   one CTA per row, online max / sum-of-exp over the shard
//   ce_grad_kernel       dlogits = (exp(l - lse) - [col == target]) * scale
//   topk_rows_kernel     per-row top-k (value desc, index asc on ties)
#include <type_traits>

#include "common.cuh"

namespace ksd8 {

constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ float ld_val(const T* p) {
  if constexpr (std::is_same<T, float>::value) return *p;
  else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
  else return __bfloat162float(*p);
}

// (m, s) <- online merge of a value v: s counts exp(v - m) for the running max m.
__device__ __forceinline__ void online_add(float& m, float& s, float v) {
  if (v > m) {
    s = s * ex2_approx((m - v) * LOG2E) + 1.f;
    m = v;
  } else {
    s += ex2_approx((v - m) * LOG2E);
  }
}

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * ex2_approx((m - m2) * LOG2E) + s2;
    m = m2;
  } else if (m2 != -INFINITY) {
    s += s2 * ex2_approx((m2 - m) * LOG2E);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ce_partials_kernel(const T* logits, int64_t V, int64_t ld,
                                                          const int64_t* targets, int64_t vstart,
                                                          float* out_max, float* out_sum,
                                                          float* out_tgt) {
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  constexpr int VEC = 16 / sizeof(T);
  const bool vec = ((reinterpret_cast<uintptr_t>(lr) & 15) == 0);
  int64_t c0 = 0;
  if (vec) {
    const int64_t nv = V / VEC;
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
      const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(lr) + i);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < VEC; ++j) online_add(m, s, ld_val(e + j));
    }
    c0 = nv * VEC;
  }
  for (int64_t c = c0 + threadIdx.x; c < V; c += blockDim.x) online_add(m, s, ld_val(lr + c));
  // block reduction of (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[8], ss[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm[0], S = ss[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) online_merge(M, S, sm[w], ss[w]);
    out_max[row] = M;
    out_sum[row] = S;
    const int64_t t = targets[row] - vstart;
    out_tgt[row] = (t >= 0 && t < V) ? ld_val(lr + t) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ce_grad_kernel(const T* logits, int64_t V, int64_t ld,
                                                      const int64_t* targets, int64_t vstart,
                                                      const float* gmax, const float* gsum,
                                                      float scale, float* dlogits,
                                                      int64_t ldd) {
  const int64_t row = blockIdx.y;
  const T* lr = logits + row * ld;
  float* dr = dlogits + row * ldd;
  // exp(l - lse) = 2^((l - max) * log2e) / sum
  const float mx = gmax[row];
  const float inv = 1.f / gsum[row];
  const int64_t t = targets[row] - vstart;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < V;
       c += (int64_t)gridDim.x * blockDim.x) {
    const float p = ex2_approx((ld_val(lr + c) - mx) * LOG2E) * inv;
    dr[c] = (p - (c == t ? 1.f : 0.f)) * scale;
  }
}

// ---------------------------------------------------------------- fused gradient + quantisation

struct CeGQArgs {
  const void* logits;
  int64_t M, V, ld;
  const int64_t* targets;
  int64_t vstart;
  const float* gmax;
  const float* gsum;
  float scale;
  int8_t* dq;          // (M, Vp) codes along the vocabulary, row stride ldq
  int64_t ldq;
  __half* dq_scales;   // (M, Vp / 128)
  int8_t* dqt;         // (V, Mp) codes along the tokens, row stride ldqt
  int64_t ldqt;
  __half* dqt_scales;  // (V, Mp / 128)
};

constexpr int CGQ_LD = 129;  // fp32 tile pitch

// One CTA per 128-token x 128-vocab tile of the logits shard.  Warp w turns
// rows 16w .. 16w + 15 into dlogits with ce_grad_kernel's expression (same
// bits), quantises each row along the vocabulary (one 128-wide group) in
// registers and parks the values in shared memory; then thread t quantises
// column t % 128 along the tokens (rows (t / 128) * 64 .. + 64, 16-byte
// stores).  Columns past V and rows past M hold zeros, so the padded tails of
// both code tensors come out zero for the GEMMs that contract over them.
template <typename T>
__global__ void __launch_bounds__(256) ce_grad_quant_kernel(CeGQArgs a) {
  extern __shared__ float gt[];  // [128][CGQ_LD]
  const int64_t r0 = (int64_t)blockIdx.y * 128, c0 = (int64_t)blockIdx.x * 128;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t vgroups = (a.V + 127) / 128;
  // per-row statistics, one row per lane (rows 16w .. 16w + 15)
  // (the target as a column of this tile, -1 when it lies elsewhere)
  float st_mx = 0.f, st_inv = 0.f;
  int st_t = -1;
  if (lane < 16 && r0 + warp * 16 + lane < a.M) {
    const int64_t r = r0 + warp * 16 + lane;
    st_mx = a.gmax[r];
    st_inv = 1.f / a.gsum[r];
    const int64_t t = a.targets[r] - a.vstart - c0;
    st_t = (t >= 0 && t < 128) ? (int)t : -1;
  }
  const int vrem = (int)min((int64_t)128, a.V - c0);  // valid columns of this tile
  const bool vec = sizeof(T) == 4 && (a.ld & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0 && c0 + 128 <= a.V;
  for (int i0 = 0; i0 < 16; i0 += 4) {
    float v[4][4];
    // the 4 rows' loads first (all in flight together)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t r = r0 + warp * 16 + i0 + u;
      const T* lr = reinterpret_cast<const T*>(a.logits) + r * a.ld;
      if (r < a.M && vec) {
        const float4 q = __ldcs(reinterpret_cast<const float4*>(lr + c0 + lane * 4));
        v[u][0] = q.x; v[u][1] = q.y; v[u][2] = q.z; v[u][3] = q.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t c = c0 + lane * 4 + j;
          v[u][j] = (r < a.M && c < a.V) ? ld_val(lr + c) : 0.f;
        }
      }
    }
    float m[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int rr = warp * 16 + i0 + u;
      const int64_t r = r0 + rr;
      const float mx = __shfl_sync(0xffffffffu, st_mx, i0 + u);
      const float inv = __shfl_sync(0xffffffffu, st_inv, i0 + u);
      const int t = __shfl_sync(0xffffffffu, st_t, i0 + u);
      const bool row_ok = r < a.M;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cl = lane * 4 + j;
        float d = 0.f;
        if (row_ok && cl < vrem) {
          const float p = ex2_approx((v[u][j] - mx) * LOG2E) * inv;
          d = (p - (cl == t ? 1.f : 0.f)) * a.scale;
        }
        v[u][j] = d;
        gt[rr * CGQ_LD + lane * 4 + j] = d;
      }
      m[u] = fmaxf(fmaxf(fabsf(v[u][0]), fabsf(v[u][1])), fmaxf(fabsf(v[u][2]), fabsf(v[u][3])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) m[u] = fmaxf(m[u], __shfl_xor_sync(0xffffffffu, m[u], o));
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t r = r0 + warp * 16 + i0 + u;
      if (r >= a.M) continue;
      __half sh;
      const float sc = gs_scale_fast(m[u], &sh);
      const float rcp = rcp_approx(sc);
      int q[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) q[j] = gs_code_fast(v[u][j], sc, rcp);
      int8_t* out = a.dq + r * a.ldq + c0 + lane * 4;
      if ((reinterpret_cast<uintptr_t>(out) & 3) == 0) {
        *reinterpret_cast<char4*>(out) = make_char4((char)q[0], (char)q[1], (char)q[2], (char)q[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) out[j] = (int8_t)q[j];
      }
      if (lane == 0) a.dq_scales[r * vgroups + blockIdx.x] = sh;
    }
  }
  __shared__ float s_amax[2][128];
  __syncthreads();
  const int cc = threadIdx.x & 127, half = threadIdx.x >> 7;
  const int64_t c = c0 + cc;
  float m = 0.f;
#pragma unroll 16
  for (int i = 0; i < 64; ++i) m = fmaxf(m, fabsf(gt[(half * 64 + i) * CGQ_LD + cc]));
  s_amax[half][cc] = m;
  __syncthreads();
  if (c >= a.V) return;
  m = fmaxf(s_amax[0][cc], s_amax[1][cc]);
  const int64_t mgroups = (a.M + 127) / 128;
  __half sh;
  const float sc = gs_scale_fast(m, &sh);
  const float rcp = rcp_approx(sc);
  int8_t* out = a.dqt + c * a.ldqt + r0 + half * 64;
  if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
#pragma unroll
    for (int q16 = 0; q16 < 4; ++q16) {
      uint32_t w[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int rr = half * 64 + q16 * 16 + jj * 4 + b;
          word |= (uint32_t)(gs_code_fast(gt[rr * CGQ_LD + cc], sc, rcp) & 0xFF) << (8 * b);
        }
        w[jj] = word;
      }
      *reinterpret_cast<uint4*>(out + q16 * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    for (int i = 0; i < 64; ++i)
      out[i] = (int8_t)gs_code_fast(gt[(half * 64 + i) * CGQ_LD + cc], sc, rcp);
  }
  if (half == 0) a.dqt_scales[c * mgroups + blockIdx.y] = sh;
}

// ---------------------------------------------------------------- top-k

constexpr int TOPK_MAX = 32;

// a before b: larger value, then smaller index
__device__ __forceinline__ bool topk_before(float va, int64_t ia, float vb, int64_t ib) {
  return va > vb || (va == vb && ia < ib);
}

template <typename T>
__global__ void __launch_bounds__(256) topk_rows_kernel(const T* vals, const int64_t* idx,
                                                        int64_t C, int64_t ld, int k,
                                                        int64_t offset, float* out_v,
                                                        int64_t* out_i) {
  const int64_t row = blockIdx.x;
  const T* vr = vals + row * ld;
  const int64_t* ir = idx ? idx + row * ld : nullptr;
  // per-thread sorted candidate list (insertion; most values fail the first test)
  float lv[TOPK_MAX];
  int64_t li[TOPK_MAX];
#pragma unroll
  for (int j = 0; j < TOPK_MAX; ++j) {
    lv[j] = -INFINITY;
    li[j] = INT64_MAX;
  }
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const float v = ld_val(vr + c);
    const int64_t id = ir ? ir[c] : offset + c;
    if (!topk_before(v, id, lv[k - 1], li[k - 1])) continue;
    // insert, keeping lv[0..k) sorted: shift the entries it beats one down
    int p = k - 1;
    bool moving = true;
#pragma unroll
    for (int q = TOPK_MAX - 1; q >= 1; --q) {
      if (q < k && moving) {
        if (topk_before(v, id, lv[q - 1], li[q - 1])) {
          lv[q] = lv[q - 1];
          li[q] = li[q - 1];
          p = q - 1;
        } else {
          moving = false;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < TOPK_MAX; ++j)
      if (j == p) {
        lv[j] = v;
        li[j] = id;
      }
  }
  // k rounds of block arg-best over the threads' list heads
  __shared__ float wv[8];
  __shared__ int64_t wi[8];
  __shared__ int wt[8];
  __shared__ int winner;
  int head = 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
#pragma unroll
    for (int j = 0; j < TOPK_MAX; ++j)
      if (j == head) {
        bv = lv[j];
        bi = li[j];
      }
    int bt = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      const int64_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      const int t2 = __shfl_xor_sync(0xffffffffu, bt, o);
      if (topk_before(v2, i2, bv, bi)) {
        bv = v2;
        bi = i2;
        bt = t2;
      }
    }
    if (lane == 0) {
      wv[warp] = bv;
      wi[warp] = bi;
      wt[warp] = bt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = wv[0];
      int64_t i = wi[0];
      int t = wt[0];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        if (topk_before(wv[w], wi[w], v, i)) {
          v = wv[w];
          i = wi[w];
          t = wt[w];
        }
      out_v[row * k + r] = v;
      out_i[row * k + r] = i;
      winner = t;
    }
    __syncthreads();
    if ((int)threadIdx.x == winner) ++head;
    __syncthreads();
  }
}

template <typename T>
static int launch_partials(const void* logits, int64_t M, int64_t V, int64_t ld,
                           const int64_t* targets, int64_t vstart, float* mx, float* sm,
                           float* tg, cudaStream_t stream) {
  ce_partials_kernel<T><<<(unsigned)M, 256, 0, stream>>>(reinterpret_cast<const T*>(logits), V,
                                                         ld, targets, vstart, mx, sm, tg);
  return KSD8_OK;
}

template <typename T>
static int launch_grad(const void* logits, int64_t M, int64_t V, int64_t ld,
                       const int64_t* targets, int64_t vstart, const float* gmax,
                       const float* gsum, float scale, float* dl, int64_t ldd,
                       cudaStream_t stream) {
  const int64_t bx = (V + 1023) / 1024;
  dim3 grid((unsigned)(bx < 64 ? bx : 64), (unsigned)M);
  ce_grad_kernel<T><<<grid, 256, 0, stream>>>(reinterpret_cast<const T*>(logits), V, ld, targets,
                                              vstart, gmax, gsum, scale, dl, ldd);
  return KSD8_OK;
}

template <typename T>
static int launch_topk(const void* vals, const int64_t* idx, int64_t M, int64_t C, int64_t ld,
                       int k, int64_t offset, float* ov, int64_t* oi, cudaStream_t stream) {
  topk_rows_kernel<T><<<(unsigned)M, 256, 0, stream>>>(reinterpret_cast<const T*>(vals), idx, C,
                                                       ld, k, offset, ov, oi);
  return KSD8_OK;
}

}  // namespace ksd8

using namespace ksd8;

int ksd8_ce_partials_launch(const void* logits, int dtype, int64_t M, int64_t V, int64_t ld,
                            const int64_t* targets, int64_t vstart, float* mx, float* sm,
                            float* tg, cudaStream_t stream) {
  if (M == 0) return KSD8_OK;
  if (dtype == KSD8_F32) return launch_partials<float>(logits, M, V, ld, targets, vstart, mx, sm, tg, stream);
  if (dtype == KSD8_BF16)
    return launch_partials<__nv_bfloat16>(logits, M, V, ld, targets, vstart, mx, sm, tg, stream);
  return launch_partials<__half>(logits, M, V, ld, targets, vstart, mx, sm, tg, stream);
}

int ksd8_ce_grad_launch(const void* logits, int dtype, int64_t M, int64_t V, int64_t ld,
                        const int64_t* targets, int64_t vstart, const float* gmax,
                        const float* gsum, float scale, float* dl, int64_t ldd,
                        cudaStream_t stream) {
  if (M == 0 || V == 0) return KSD8_OK;
  if (dtype == KSD8_F32)
    return launch_grad<float>(logits, M, V, ld, targets, vstart, gmax, gsum, scale, dl, ldd, stream);
  if (dtype == KSD8_BF16)
    return launch_grad<__nv_bfloat16>(logits, M, V, ld, targets, vstart, gmax, gsum, scale, dl,
                                      ldd, stream);
  return launch_grad<__half>(logits, M, V, ld, targets, vstart, gmax, gsum, scale, dl, ldd, stream);
}

int ksd8_ce_grad_quant_launch(const void* logits, int dtype, int64_t M, int64_t V, int64_t ld,
                              const int64_t* targets, int64_t vstart, const float* gmax,
                              const float* gsum, float scale, int8_t* dq, int64_t ldq,
                              void* dq_scales, int8_t* dqt, int64_t ldqt, void* dqt_scales,
                              cudaStream_t stream) {
  if (M == 0 || V == 0) return KSD8_OK;
  CeGQArgs a;
  a.logits = logits; a.M = M; a.V = V; a.ld = ld; a.targets = targets; a.vstart = vstart;
  a.gmax = gmax; a.gsum = gsum; a.scale = scale; a.dq = dq; a.ldq = ldq;
  a.dq_scales = reinterpret_cast<__half*>(dq_scales); a.dqt = dqt; a.ldqt = ldqt;
  a.dqt_scales = reinterpret_cast<__half*>(dqt_scales);
  const int smem = 128 * CGQ_LD * 4;
  static unsigned attr = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr & (1u << dev))) {
    cudaFuncSetAttribute(ce_grad_quant_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(ce_grad_quant_kernel<__nv_bfloat16>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(ce_grad_quant_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr |= (1u << dev);
  }
  dim3 grid((unsigned)((V + 127) / 128), (unsigned)((M + 127) / 128));
  if (dtype == KSD8_F32) ce_grad_quant_kernel<float><<<grid, 256, smem, stream>>>(a);
  else if (dtype == KSD8_BF16) ce_grad_quant_kernel<__nv_bfloat16><<<grid, 256, smem, stream>>>(a);
  else ce_grad_quant_kernel<__half><<<grid, 256, smem, stream>>>(a);
  return KSD8_OK;
}

int ksd8_topk_rows_launch(const void* vals, int dtype, const int64_t* idx, int64_t M, int64_t C,
                          int64_t ld, int k, int64_t offset, float* ov, int64_t* oi,
                          cudaStream_t stream) {
  if (M == 0) return KSD8_OK;
  if (dtype == KSD8_F32) return launch_topk<float>(vals, idx, M, C, ld, k, offset, ov, oi, stream);
  if (dtype == KSD8_BF16)
    return launch_topk<__nv_bfloat16>(vals, idx, M, C, ld, k, offset, ov, oi, stream);
  return launch_topk<__half>(vals, idx, M, C, ld, k, offset, ov, oi, stream);
}
