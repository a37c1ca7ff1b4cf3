// Incremental Rosa matching for drafting (config 5): the answer of
// _match_payload_sign (ksdraft/model/rosa.py:40-98) at new positions appended
// to a long context, without re-matching the context.
//
// The reference only matches whole sequences.  Its result at position t
// depends on the q bits up to t and on the (k, v) bits up to t, so appending
// positions leaves every earlier answer unchanged; a decode step therefore
// only answers the new positions, against every key j <= t - 1, with the
// same semantics as the sequence matchers of rosa.cu (64-bit windows W(t),
// bit 63 = x[t]; common-suffix length clz(Wq ^ Wk), capped at
// min(max_len, t) and at j + 1; the latest j among the longest; sign from
// v[j + 1]).  For sequences of at least max_len + 1 positions the cap
// min(62, T - 1) of the reference is the constant max_len = 62.
//
// Per stream the keys are split three ways:
//   early keys   j < r0 = max_len - 1: their windows reach before position 0,
//                so their length is also capped at j + 1; matched directly,
//                bit-parallel over their k word (see the step kernel);
//   main run     r0 <= j < n_main: sorted by (W(j), j) once (decode_build),
//                static until the next rebuild -- the longest match against
//                them is reached at the query's sorted neighbours, the latest
//                endpoint sharing that prefix is a range maximum over ranks
//                (max of j + 1 per block of 64 ranks plus the partial blocks);
//   delta        n_main <= j <= t - 1: the keys appended since the last
//                build, matched directly and bit-parallel per k word (the
//                caller rebuilds the main run when the delta grows past its
//                budget).
// All three give exact (length, latest j) candidates; the best of them is the
// sequence matcher's answer.
#include "common.cuh"

namespace ksd8 {

namespace {

constexpr int DEC_BLK = 64;        // ranks per range-maximum block
constexpr int DEC_WARPS = 8;       // streams per CTA in the step kernel
constexpr int DEC_MAX_NEW = 32;    // new positions per step
constexpr int DEC_MAX_TOP = 512;   // sampled windows of the main run held in shared memory
constexpr int DEC_DELTA_WORDS = 34;  // k words of the delta region held in shared memory
constexpr int DEC_SUB = 8;         // ranks per inner sample

// Sample index of a main run, per row (stride dec_smp_stride(cap) uint64):
// [0, cap / DEC_BLK): the windows of ranks 0, DEC_BLK, 2 DEC_BLK, ...;
// then [cap / DEC_BLK, + cap / DEC_SUB): the windows of ranks 0, DEC_SUB, ...
// Both contiguous, so the step kernel's per-row sample load and the inner
// samples of a block are whole sectors.
__host__ __device__ constexpr int64_t dec_smp_stride(int64_t cap) {
  return cap / DEC_BLK + cap / DEC_SUB;
}

// window of position t from bit words w (global or shared), bits before 0 are 0
__device__ __forceinline__ uint64_t window_at(const uint64_t* w, int64_t t) {
  const int64_t wi = t >> 6;
  const int sh = (int)(t & 63) + 1;
  const uint64_t hi = w[wi];
  const uint64_t lo = wi > 0 ? w[wi - 1] : 0ull;
  return sh == 64 ? hi : ((lo >> sh) | (hi << (64 - sh)));
}

__device__ __forceinline__ int lcp64(uint64_t a, uint64_t b) {
  const uint64_t x = a ^ b;
  return x ? __clzll((long long)x) : 64;
}

// (W, j) order of the main run
__device__ __forceinline__ bool key_less(uint64_t wa, uint32_t ja, uint64_t wb, uint32_t jb) {
  return wa < wb || (wa == wb && ja < jb);
}

// candidate (len, j) is better than (best, bestj): longer, or as long and later
__device__ __forceinline__ bool better(int len, int64_t j, int best, int64_t bestj) {
  return len > best || (len == best && len > 0 && j > bestj);
}

}  // namespace

// ---------------------------------------------------------------- build
//
// One CTA per stream: the windows of keys j in [r0, n_keys) are sorted by
// (W(j), j) with a bitonic sort in shared memory; sw / sj receive the sorted
// windows and positions (row stride cap), blk the maximum of j + 1 per block
// of DEC_BLK ranks (row stride cap / DEC_BLK).
__global__ void __launch_bounds__(256) rosa_decode_build_kernel(const uint64_t* __restrict__ kw,
                                                                int64_t nw, int64_t n_keys,
                                                                int r0, int np, int64_t cap,
                                                                uint64_t* __restrict__ sw,
                                                                uint16_t* __restrict__ sj,
                                                                uint16_t* __restrict__ blk,
                                                                uint64_t* __restrict__ smp) {
  extern __shared__ __align__(16) uint8_t dsm[];
  uint64_t* W = reinterpret_cast<uint64_t*>(dsm);
  uint32_t* J = reinterpret_cast<uint32_t*>(W + np);
  uint64_t* bits = reinterpret_cast<uint64_t*>(J + np + (np & 1));
  const int64_t stream = blockIdx.x;
  const int64_t nk = n_keys > r0 ? n_keys - r0 : 0;
  const int64_t words = (n_keys + 63) / 64;
  for (int64_t i = threadIdx.x; i < words; i += blockDim.x) bits[i] = kw[stream * nw + i];
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    const bool real = i < nk;
    W[i] = real ? window_at(bits, r0 + i) : ~0ull;
    J[i] = real ? (uint32_t)(r0 + i) : 0xFFFFFFFFu;
  }
  __syncthreads();
  for (int k = 2; k <= np; k <<= 1) {
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int pr = threadIdx.x; pr < (np >> 1); pr += blockDim.x) {   // pairs (i, i + jj)
        const int i = ((pr & ~(jj - 1)) << 1) | (pr & (jj - 1));
        const int l = i | jj;
        const bool up = (i & k) == 0;
        const uint64_t wi = W[i], wl = W[l];
        const uint32_t ji = J[i], jl = J[l];
        if (key_less(wl, jl, wi, ji) == up) {
          W[i] = wl; W[l] = wi;
          J[i] = jl; J[l] = ji;
        }
      }
      __syncthreads();
    }
  }
  for (int64_t r = threadIdx.x; r < nk; r += blockDim.x) {
    sw[stream * cap + r] = W[r];
    sj[stream * cap + r] = (uint16_t)J[r];
  }
  {
    uint64_t* sr = smp + stream * dec_smp_stride(cap);
    for (int64_t b = threadIdx.x; b * DEC_BLK < nk; b += blockDim.x) sr[b] = W[b * DEC_BLK];
    for (int64_t q = threadIdx.x; q * DEC_SUB < nk; q += blockDim.x)
      sr[cap / DEC_BLK + q] = W[q * DEC_SUB];
  }
  const int64_t nb = (nk + DEC_BLK - 1) / DEC_BLK;
  for (int64_t b = threadIdx.x; b < nb; b += blockDim.x) {
    uint32_t m = 0;
    const int64_t e = min(nk, (b + 1) * DEC_BLK);
    for (int64_t r = b * DEC_BLK; r < e; ++r) m = max(m, J[r] + 1u);
    blk[stream * (cap / DEC_BLK) + b] = (uint16_t)m;
  }
}

// ---------------------------------------------------------------- merge
//
// Rebuild by merging: the keys appended since the last build, j in
// [max(n_old, r0), n_new), are sorted in shared memory and merged with the old
// main run (sw_in, sj_in: keys r0 .. n_old - 1): an old key moves up by the
// number of new keys with a smaller window (a new key's position is larger,
// so on equal windows the old key comes first), a new key lands at its own
// rank plus the number of old keys with a window <= its own.  One CTA per
// stream; O((n_old + nd) log nd) instead of re-sorting the whole run.
__global__ void __launch_bounds__(256) rosa_decode_merge_kernel(
    const uint64_t* __restrict__ kw, int64_t nw, int64_t n_old, int64_t n_new, int r0, int npd,
    int64_t cap, const uint64_t* __restrict__ sw_in, const uint16_t* __restrict__ sj_in,
    uint64_t* __restrict__ sw, uint16_t* __restrict__ sj, uint16_t* __restrict__ blk,
    uint64_t* __restrict__ smp) {
  extern __shared__ __align__(16) uint8_t dsm[];
  uint64_t* W = reinterpret_cast<uint64_t*>(dsm);
  uint32_t* J = reinterpret_cast<uint32_t*>(W + npd);
  uint64_t* bits = reinterpret_cast<uint64_t*>(J + npd + (npd & 1));
  const int64_t stream = blockIdx.x;
  const int64_t nk_old = n_old > r0 ? n_old - r0 : 0;
  const int64_t dlo = max(n_old, (int64_t)r0);
  const int64_t nd = n_new > dlo ? n_new - dlo : 0;
  const int64_t w0 = dlo > 63 ? (dlo >> 6) - 1 : 0;
  const int64_t nwd = nd > 0 ? ((n_new - 1) >> 6) - w0 + 1 : 0;
  for (int64_t i = threadIdx.x; i < nwd; i += blockDim.x) bits[i] = kw[stream * nw + w0 + i];
  __syncthreads();
  for (int i = threadIdx.x; i < npd; i += blockDim.x) {
    const bool real = i < nd;
    uint64_t w = ~0ull;
    if (real) {
      const int64_t j = dlo + i;
      const int64_t wi = (j >> 6) - w0;
      const int sh = (int)(j & 63) + 1;
      const uint64_t h = bits[wi];
      const uint64_t l0 = (j >> 6) > 0 ? bits[wi - 1] : 0ull;
      w = sh == 64 ? h : ((l0 >> sh) | (h << (64 - sh)));
    }
    W[i] = w;
    J[i] = real ? (uint32_t)(dlo + i) : 0xFFFFFFFFu;
  }
  __syncthreads();
  for (int k = 2; k <= npd; k <<= 1) {
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int pr = threadIdx.x; pr < (npd >> 1); pr += blockDim.x) {   // pairs (i, i + jj)
        const int i = ((pr & ~(jj - 1)) << 1) | (pr & (jj - 1));
        const int l = i | jj;
        const bool up = (i & k) == 0;
        const uint64_t wi = W[i], wl = W[l];
        const uint32_t ji = J[i], jl = J[l];
        if (key_less(wl, jl, wi, ji) == up) {
          W[i] = wl; W[l] = wi;
          J[i] = jl; J[l] = ji;
        }
      }
      __syncthreads();
    }
  }
  const uint64_t* swi = sw_in + stream * cap;
  const uint16_t* sji = sj_in + stream * cap;
  uint64_t* swo = sw + stream * cap;
  uint16_t* sjo = sj + stream * cap;
  for (int64_t r = threadIdx.x; r < nk_old; r += blockDim.x) {
    const uint64_t w = swi[r];
    int64_t a = 0, b = nd;   // new keys with a window < w
    while (a < b) {
      const int64_t mid = (a + b) >> 1;
      if (W[mid] < w) a = mid + 1; else b = mid;
    }
    swo[r + a] = w;
    sjo[r + a] = sji[r];
  }
  for (int64_t i = threadIdx.x; i < nd; i += blockDim.x) {
    const uint64_t w = W[i];
    int64_t a = 0, b = nk_old;   // old keys with a window <= w
    while (a < b) {
      const int64_t mid = (a + b) >> 1;
      if (swi[mid] <= w) a = mid + 1; else b = mid;
    }
    swo[i + a] = w;
    sjo[i + a] = (uint16_t)J[i];
  }
  __syncthreads();
  const int64_t nk = nk_old + nd;
  {
    uint64_t* sr = smp + stream * dec_smp_stride(cap);
    for (int64_t b = threadIdx.x; b * DEC_BLK < nk; b += blockDim.x) sr[b] = swo[b * DEC_BLK];
    for (int64_t q = threadIdx.x; q * DEC_SUB < nk; q += blockDim.x)
      sr[cap / DEC_BLK + q] = swo[q * DEC_SUB];
  }
  const int64_t nb = (nk + DEC_BLK - 1) / DEC_BLK;
  for (int64_t bb = threadIdx.x; bb < nb; bb += blockDim.x) {
    uint32_t m = 0;
    const int64_t e = min(nk, (bb + 1) * DEC_BLK);
    for (int64_t r = bb * DEC_BLK; r < e; ++r) m = max(m, (uint32_t)sjo[r] + 1u);
    blk[stream * (cap / DEC_BLK) + bb] = (uint16_t)m;
  }
}

// ---------------------------------------------------------------- step

namespace {

// first rank r in [0, nk) with SW[r] >= key (nk when none): the block
// samples top[b] = SW[b * DEC_BLK] (shared memory) pick the block, its 7 inner
// samples SW[base + 8i] (contiguous in the sample index, sub) pick the run of
// 8, whose 7 remaining windows give the rank: two rounds of independent loads
// of 56 contiguous bytes each.
__device__ __forceinline__ int64_t main_lower_bound(const uint64_t* top, int ntop,
                                                    const uint64_t* sub, const uint64_t* swr,
                                                    int64_t nk, uint64_t key) {
  int lo = 0, hi = ntop;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (top[mid] < key) lo = mid + 1; else hi = mid;
  }
  if (lo == 0) return 0;
  // SW[base] < key; the answer lies in [base + 1, end]
  const int64_t base = (int64_t)(lo - 1) * DEC_BLK;
  const int64_t end = min(nk, (int64_t)lo * DEC_BLK);
  static_assert(DEC_BLK == 8 * DEC_SUB && DEC_SUB == 8, "two rounds of 8");
  uint64_t v[7];
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    const int64_t r = base + DEC_SUB * (i + 1);
    v[i] = r < end ? sub[r / DEC_SUB] : ~0ull;
  }
  int c = 0;  // inner samples < key, i = 1 .. 7 (a prefix: the run is sorted)
#pragma unroll
  for (int i = 0; i < 7; ++i) c += (base + DEC_SUB * (i + 1) < end && v[i] < key) ? 1 : 0;
  const int64_t b8 = base + DEC_SUB * c;  // SW[b8] < key
#pragma unroll
  for (int i = 0; i < 7; ++i) {
    const int64_t r = b8 + 1 + i;
    v[i] = r < end ? swr[r] : ~0ull;
  }
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < 7; ++i) cnt += (b8 + 1 + i < end && v[i] < key) ? 1 : 0;
  return b8 + 1 + cnt;
}

}  // namespace

struct DecodeArgs {
  const void* proj[3];   // q, k, v projections (contexts, k_new, streams); null: the
                         // bits of the new positions are already in the histories
  int dtype;
  int64_t contexts, streams, k_new, t0, n_main;
  const int64_t* pos;    // device [t0, n_main] overriding the two scalars (CUDA graphs)
  int max_len;
  uint64_t* bits[3];     // q, k, v bit histories (contexts * streams, nw)
  int64_t nw;
  const uint64_t* sw;    // main run windows (contexts * streams, cap)
  const uint16_t* sj;    // main run positions
  const uint16_t* blk;   // max(j + 1) per DEC_BLK ranks (contexts * streams, cap / DEC_BLK)
  const uint64_t* smp;   // sample index (contexts * streams, dec_smp_stride(cap))
  int64_t cap;
  const float* payload;  // (streams) or null
  void* out;             // out[c * out_cs + i * streams + s] for new position i
  int64_t out_cs;
  int out_dtype;
  int32_t* match_len;    // match_len[row * ml_rs + i], or null
  int32_t* match_end;
  int64_t ml_rs;
};

template <typename T> __device__ __forceinline__ float as_float(T v);
template <> __device__ __forceinline__ float as_float<float>(float v) { return v; }
template <> __device__ __forceinline__ float as_float<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float as_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ bool proj_positive(const void* p, int64_t i) {
  return as_float<T>(reinterpret_cast<const T*>(p)[i]) > 0.f;
}

__global__ void __launch_bounds__(DEC_WARPS * 32) rosa_decode_step_kernel(DecodeArgs a) {
  __shared__ uint64_t top_all[DEC_WARPS][DEC_MAX_TOP];
  __shared__ uint64_t dwords_all[DEC_WARPS][DEC_DELTA_WORDS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t st = (int64_t)blockIdx.x * DEC_WARPS + warp;
  if (st >= a.contexts * a.streams) return;  // whole warp; no CTA barrier below
  const unsigned full = 0xffffffffu;
  const int64_t c = st / a.streams, s = st % a.streams;
  const int K = (int)a.k_new;
  const int64_t t0 = a.pos ? a.pos[0] : a.t0;
  const int64_t n_main = a.pos ? a.pos[1] : a.n_main;
  uint64_t* top = top_all[warp];
  uint64_t* dwords = dwords_all[warp];

  // 1. append the new bits (proj > 0, rosa.py:156-158) at positions t0 .. t0 + K - 1
  const bool append = a.proj[0] != nullptr;
  unsigned m[3] = {0u, 0u, 0u};
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    bool bit = false;
    if (append && lane < K) {
      const int64_t i = (c * a.k_new + lane) * a.streams + s;
      switch (a.dtype) {
        case KSD8_F32: bit = proj_positive<float>(a.proj[q], i); break;
        case KSD8_BF16: bit = proj_positive<__nv_bfloat16>(a.proj[q], i); break;
        default: bit = proj_positive<__half>(a.proj[q], i); break;
      }
    }
    m[q] = __ballot_sync(full, bit);
  }
  if (append && lane == 0) {
    const int64_t wi = t0 >> 6;
    const int off = (int)(t0 & 63);
    const uint64_t M = (K == 64) ? ~0ull : ((1ull << K) - 1ull);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      uint64_t* w = a.bits[q] + st * a.nw;
      w[wi] = (w[wi] & ~(M << off)) | ((uint64_t)m[q] << off);
      if (off + K > 64) {
        const int rs = 64 - off;
        w[wi + 1] = (w[wi + 1] & ~(M >> rs)) | ((uint64_t)m[q] >> rs);
      }
    }
  }
  __syncwarp();

  const uint64_t* qrow = a.bits[0] + st * a.nw;
  const uint64_t* krow = a.bits[1] + st * a.nw;
  const uint64_t* vrow = a.bits[2] + st * a.nw;
  const int r0 = a.max_len > 0 ? a.max_len - 1 : 0;
  const int64_t nk = n_main > r0 ? n_main - r0 : 0;     // main run size
  const int ntop = (int)((nk + DEC_BLK - 1) / DEC_BLK);
  const uint64_t* swr = a.sw + st * a.cap;
  const uint16_t* sjr = a.sj + st * a.cap;
  const uint16_t* blkr = a.blk + st * (a.cap / DEC_BLK);
  const uint64_t* smr = a.smp + st * dec_smp_stride(a.cap);
  const uint64_t* subr = smr + a.cap / DEC_BLK;
  for (int b = lane; b < ntop; b += 32) top[b] = smr[b];
  // delta keys j in [dlo, t0 + K - 2]; their windows read words w0 .. of k
  const int64_t dlo = max(n_main, (int64_t)r0);
  const int64_t dhi = t0 + K - 2;
  const int64_t w0 = dlo > 63 ? (dlo >> 6) - 1 : 0;
  if (dhi >= dlo) {
    const int64_t nwd = (dhi >> 6) - w0 + 1;
    for (int64_t i = lane; i < nwd; i += 32) dwords[i] = krow[w0 + i];
  }
  const uint64_t kw0 = krow[0];  // every early key's window lies in word 0
  __syncwarp();

  // 2. main run, one query per lane: longest match at the sorted neighbours,
  //    then the rank interval sharing that prefix
  const int64_t t = t0 + lane;
  const bool valid = lane < K;
  const uint64_t wq = valid ? window_at(qrow, t) : 0ull;
  const int capq = valid ? (int)min((int64_t)a.max_len, t) : 0;
  int Lm = 0;
  int64_t lo = 0, hi = 0;
  if (valid && nk > 0 && capq > 0) {
    const int64_t r = main_lower_bound(top, ntop, subr, swr, nk, wq);
    int lraw = 0;
    if (r > 0) lraw = lcp64(wq, swr[r - 1]);
    if (r < nk) lraw = max(lraw, lcp64(wq, swr[r]));
    Lm = min(lraw, capq);
    if (Lm > 0) {
      const uint64_t pre = Lm >= 64 ? wq : (wq >> (64 - Lm)) << (64 - Lm);
      const uint64_t last = Lm >= 64 ? wq : pre | (~0ull >> Lm);
      lo = main_lower_bound(top, ntop, subr, swr, nk, pre);
      hi = last == ~0ull ? nk : main_lower_bound(top, ntop, subr, swr, nk, last + 1);
    }
  }

  // 3a. per query, the warp together: the latest endpoint in [lo, hi) of the
  //     main run (partial blocks and block maxima).  Candidates are packed as
  //     (length << 32) | (j + 1): the larger packed value is the longer match,
  //     then the later endpoint.
  unsigned long long mine = 0ull;  // lane i: the best candidate of query i so far
  for (int i = 0; i < K; ++i) {
    const int L = __shfl_sync(full, Lm, i);
    if (L == 0) continue;  // uniform across the warp
    const int64_t ilo = __shfl_sync(full, lo, i), ihi = __shfl_sync(full, hi, i);
    uint32_t mx = 0;
    const int64_t b0 = (ilo + DEC_BLK - 1) / DEC_BLK, b1 = ihi / DEC_BLK;
    if (b0 >= b1) {
      for (int64_t r = ilo + lane; r < ihi; r += 32) mx = max(mx, (uint32_t)sjr[r] + 1u);
    } else {
      for (int64_t r = ilo + lane; r < b0 * DEC_BLK; r += 32)
        mx = max(mx, (uint32_t)sjr[r] + 1u);
      for (int64_t r = b1 * DEC_BLK + lane; r < ihi; r += 32)
        mx = max(mx, (uint32_t)sjr[r] + 1u);
      for (int64_t b = b0 + lane; b < b1; b += 32) mx = max(mx, (uint32_t)blkr[b]);
    }
    mx = __reduce_max_sync(full, mx);
    if (lane == i) mine = ((unsigned long long)L << 32) | mx;
  }

  // 3b. early keys (j < r0: also capped at j + 1) and delta keys (dlo <= j <=
  //     t - 1), bit-parallel over the 64 keys of a k word: the keys whose
  //     windows agree with the query window in the top l bits are a bit mask
  //     M_l = M_{l-1} & (k shifted by l == q[t - l]), so a word costs one
  //     and-step per matched bit (about log2 of the keys scanned), and the
  //     latest key of the longest match is the highest bit of the last
  //     non-empty mask.  8 queries at a time, 4 lanes per query taking every
  //     4th word; item -1 of a query is the early-key word.
  for (int c0 = 0; c0 < K; c0 += 8) {
    const int ql = lane >> 2, sub = lane & 3;
    const int qi = c0 + ql;                     // this lane's query
    const bool qok = qi < K;
    const uint64_t qv = __shfl_sync(full, wq, qok ? qi : 0);
    const int qcap_src = __shfl_sync(full, capq, qok ? qi : 0);
    const int qcap = qok ? qcap_src : 0;
    const int64_t tq = t0 + qi;
    unsigned long long pk = 0ull;
    if (qok && qcap > 0) {
      const int64_t wlo = dlo >> 6, whi = (tq - 1) >> 6;   // delta words of this query
      for (int64_t w = wlo - 1 + sub; w <= whi; w += 4) {
        uint64_t kwd, kprev, M;
        bool early;
        int64_t jb;
        if (w == wlo - 1) {                      // the early keys j < min(r0, t)
          const int64_t ne = min((int64_t)r0, tq);
          if (ne <= 0) continue;
          kwd = kw0;
          kprev = 0ull;
          M = ne >= 64 ? ~0ull : ((1ull << ne) - 1ull);
          early = true;
          jb = 0;
        } else {
          if (tq - 1 < dlo) continue;            // no delta keys for this query
          kwd = dwords[w - w0];
          kprev = w > 0 ? dwords[w - 1 - w0] : 0ull;
          const int64_t lo_b = max(dlo - (w << 6), (int64_t)0);
          const int64_t hi_b = min(tq - 1 - (w << 6), (int64_t)63);
          if (lo_b > hi_b) continue;
          M = (~0ull << lo_b) & (~0ull >> (63 - hi_b));
          early = false;
          jb = w << 6;
        }
        int len = 0;
        while (len < qcap) {
          const uint64_t sh = len ? ((kwd << len) | (kprev >> (64 - len))) : kwd;
          uint64_t e = ((qv >> (63 - len)) & 1ull) ? sh : ~sh;
          if (early) e &= ~0ull << len;          // length <= j + 1
          const uint64_t m2 = M & e;
          if (!m2) break;
          M = m2;
          ++len;
        }
        if (len > 0) {
          const unsigned long long c =
              ((unsigned long long)len << 32) | (unsigned long long)(jb + 63 - __clzll((long long)M) + 1);
          pk = c > pk ? c : pk;
        }
      }
    }
    // the 4 lanes of a query, then its owner lane
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      const unsigned long long other = __shfl_xor_sync(full, pk, o);
      pk = other > pk ? other : pk;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const unsigned long long v = __shfl_sync(full, pk, 4 * q);
      if (lane == c0 + q && v > mine) mine = v;
    }
  }
  const int best = (int)(mine >> 32);
  const int64_t bestj = mine ? (int64_t)(mine & 0xFFFFFFFFull) - 1 : -1;

  // 4. sign from v[j + 1], payload, outputs
  if (valid) {
    float sign = -1.f;
    if (bestj >= 0) {
      const int64_t succ = bestj + 1;
      sign = ((vrow[succ >> 6] >> (succ & 63)) & 1ull) ? 1.f : -1.f;
    }
    const float o = (a.payload ? a.payload[s] : 1.f) * sign;
    const int64_t oo = c * a.out_cs + lane * a.streams + s;
    if (a.out_dtype == KSD8_F32)
      reinterpret_cast<float*>(a.out)[oo] = o;
    else if (a.out_dtype == KSD8_BF16)
      reinterpret_cast<__nv_bfloat16*>(a.out)[oo] = __float2bfloat16_rn(o);
    else
      reinterpret_cast<__half*>(a.out)[oo] = __float2half_rn(o);
    if (a.match_len) a.match_len[st * a.ml_rs + lane] = best;
    if (a.match_end) a.match_end[st * a.ml_rs + lane] = (int32_t)bestj;
  }
}

}  // namespace ksd8

using namespace ksd8;

int ksd8_rosa_decode_build_launch(const uint64_t* kw, int64_t n_streams, int64_t nw,
                                  int64_t n_keys, int max_len, uint64_t* sw, uint16_t* sj,
                                  uint16_t* blk, uint64_t* smp, int64_t cap,
                                  cudaStream_t stream) {
  if (n_streams == 0) return KSD8_OK;
  const int r0 = max_len > 0 ? max_len - 1 : 0;
  const int64_t nk = n_keys > r0 ? n_keys - r0 : 0;
  if (nk == 0) return KSD8_OK;
  int np = 1;
  while (np < nk) np <<= 1;
  const size_t smem = (size_t)np * 12 + 8 + (size_t)((n_keys + 63) / 64) * 8;
  if (smem > 227 * 1024) return KSD8_ERR_UNSUPPORTED;
  static unsigned attr_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 32) return KSD8_ERR_UNSUPPORTED;
  if (!(attr_done & (1u << dev))) {
    if (cudaFuncSetAttribute(rosa_decode_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    attr_done |= 1u << dev;
  }
  rosa_decode_build_kernel<<<(unsigned)n_streams, 256, smem, stream>>>(kw, nw, n_keys, r0, np,
                                                                       cap, sw, sj, blk, smp);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

int ksd8_rosa_decode_step_launch(const void* const* proj, int dtype, int64_t contexts,
                                 int64_t streams, int64_t k_new, int64_t t0, int64_t n_main,
                                 int max_len, uint64_t* const* bits, int64_t nw,
                                 const uint64_t* sw, const uint16_t* sj, const uint16_t* blk,
                                 const uint64_t* smp, int64_t cap, const float* payload, void* out, int64_t out_cs,
                                 int out_dtype, int32_t* match_len, int32_t* match_end,
                                 int64_t ml_rs, const int64_t* pos, cudaStream_t stream) {
  DecodeArgs a;
  for (int q = 0; q < 3; ++q) {
    a.proj[q] = proj[q];
    a.bits[q] = bits[q];
  }
  a.dtype = dtype;
  a.contexts = contexts; a.streams = streams; a.k_new = k_new; a.t0 = t0; a.n_main = n_main;
  a.pos = pos;
  a.max_len = max_len; a.nw = nw; a.sw = sw; a.sj = sj; a.blk = blk; a.smp = smp; a.cap = cap;
  a.payload = payload; a.out = out; a.out_cs = out_cs; a.out_dtype = out_dtype;
  a.match_len = match_len; a.match_end = match_end; a.ml_rs = ml_rs;
  const int64_t n = contexts * streams;
  if (n == 0 || k_new == 0) return KSD8_OK;
  rosa_decode_step_kernel<<<(unsigned)((n + DEC_WARPS - 1) / DEC_WARPS), DEC_WARPS * 32, 0,
                            stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

int ksd8_rosa_decode_merge_launch(const uint64_t* kw, int64_t n_streams, int64_t nw,
                                  int64_t n_old, int64_t n_new, int max_len,
                                  const uint64_t* sw_in, const uint16_t* sj_in, uint64_t* sw,
                                  uint16_t* sj, uint16_t* blk, uint64_t* smp, int64_t cap,
                                  cudaStream_t stream) {
  if (n_streams == 0) return KSD8_OK;
  const int r0 = max_len > 0 ? max_len - 1 : 0;
  const int64_t dlo = n_old > r0 ? n_old : r0;
  const int64_t nd = n_new > dlo ? n_new - dlo : 0;
  int npd = 1;
  while (npd < nd) npd <<= 1;
  const int64_t w0 = dlo > 63 ? (dlo >> 6) - 1 : 0;
  const int64_t nwd = nd > 0 ? ((n_new - 1) >> 6) - w0 + 1 : 0;
  const size_t smem = (size_t)npd * 12 + 8 + (size_t)nwd * 8;
  if (smem > 100 * 1024) return KSD8_ERR_UNSUPPORTED;
  static unsigned attr_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 32) return KSD8_ERR_UNSUPPORTED;
  if (!(attr_done & (1u << dev))) {
    if (cudaFuncSetAttribute(rosa_decode_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             100 * 1024) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    attr_done |= 1u << dev;
  }
  rosa_decode_merge_kernel<<<(unsigned)n_streams, 256, smem, stream>>>(
      kw, nw, n_old, n_new, r0, npd, cap, sw_in, sj_in, sw, sj, blk, smp);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

// host-side limits of the step kernel (shared with the C ABI checks)
int ksd8_rosa_decode_limits(int64_t* max_new, int64_t* max_main, int64_t* max_delta_words) {
  *max_new = DEC_MAX_NEW;
  *max_main = (int64_t)DEC_MAX_TOP * DEC_BLK;
  *max_delta_words = DEC_DELTA_WORDS;
  return KSD8_OK;
}
