// Rosa 1-bit hard-retrieval mixer kernels (ksdraft/model/rosa.py).
//
//  rosa_pack_bits_kernel   bits = x > 0 packed 64 per word, per stream
//                          (rosa.py:156-158 and the int8 inputs of :40).
//  rosa_match_kernel       _match_payload_sign (rosa.py:40-98): for every t the
//                          longest suffix match L <= max_len (the reference's
//                          62-bit cap is part of the semantics) against key
//                          suffixes ending at j in [L-1, t-1], the latest such j,
//                          sign = v[j+1] ? +1 : -1, -1 without a match; the
//                          payload multiply of :164 is fused into the store.
//  rosa_timemix_quant_kernel _shifted (rosa.py:128-133) fused with the per-token
//                          GS128 quantisation Int8Linear.forward applies to the
//                          q/k/v projection inputs (linear.py:69).
//
// Match algorithm: the 64 most recent bits ending at t form a window word
// W(t) with bit 63 = x[t], bit 62 = x[t-1], ...; the common-suffix length of
// q at t and k at j is clz(Wq(t) ^ Wk(j)), capped at min(max_len, j+1).  One
// CTA owns one stream: all key windows Wk(j) sit in shared memory, a warp
// owns 32 consecutive positions t and walks j downwards in lockstep so the
// Wk(j) reads are broadcasts.  The first j that reaches a length is the
// latest one, so only strictly longer matches replace the current best;
// a lane stops once best == min(max_len, t) and the warp stops when no lane
// can still improve (remaining j are too short: length <= j+1).
#include <cstdlib>

#include "common.cuh"

namespace ksd8 {

template <typename T>
__device__ __forceinline__ bool positive(T v);
template <>
__device__ __forceinline__ bool positive<float>(float v) { return v > 0.f; }
template <>
__device__ __forceinline__ bool positive<__half>(__half v) { return __half2float(v) > 0.f; }
template <>
__device__ __forceinline__ bool positive<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v) > 0.f;
}
template <>
__device__ __forceinline__ bool positive<int8_t>(int8_t v) { return v > 0; }

// One thread per (word, stream); consecutive threads take consecutive streams
// so that reads of a (B, T, S) layout are coalesced along S.
template <typename T>
__global__ void rosa_pack_bits_kernel(const T* x, int64_t batch, int64_t t_len, int64_t streams,
                                      int64_t sb, int64_t st, int64_t ss, uint64_t* words) {
  const int64_t nw = (t_len + 63) / 64;
  const int64_t total = batch * streams * nw;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i % streams;
    const int64_t rest = i / streams;
    const int64_t w = rest % nw;
    const int64_t b = rest / nw;
    const T* base = x + b * sb + s * ss;
    uint64_t word = 0;
    const int64_t t0 = w * 64;
    const int n = (int)min((int64_t)64, t_len - t0);
    for (int k = 0; k < n; ++k)
      if (positive<T>(base[(t0 + k) * st])) word |= (1ull << k);
    words[((b * streams + s) * nw) + w] = word;
  }
}

// W(t): bits x[t-63 .. t], x[t] at bit 63; positions before 0 read as 0.
__device__ __forceinline__ uint64_t window_at(const uint64_t* w, int64_t t) {
  const int64_t wi = t >> 6;
  const int sh = (int)(t & 63) + 1;  // 1..64
  const uint64_t hi = w[wi];
  const uint64_t lo = wi > 0 ? w[wi - 1] : 0ull;
  return sh == 64 ? hi : ((lo >> sh) | (hi << (64 - sh)));
}

struct MatchArgs {
  const uint64_t* qw;
  const uint64_t* kw;
  const uint64_t* vw;
  int64_t batch, streams, t_len;
  int max_len;
  const float* payload;
  void* out;
  int out_dtype;
  int64_t ob, ot, os;
  int32_t* match_len;
  int32_t* match_end;
  // adaptive matching: the chunked kernel hands a stream whose level-12 chain
  // walks exceed the budget to the sorted kernel through redo = [count, ids...]
  int32_t* redo;
  int redo_budget;  // chain steps per position allowed on average
  int redo_pass;    // 1: the sorted kernel runs only the listed streams
};

__global__ void __launch_bounds__(512) rosa_match_kernel(MatchArgs a) {
  extern __shared__ uint64_t sk[];  // Wk(j), j = 0 .. T-1
  const int64_t stream = blockIdx.x;
  const int64_t T = a.t_len;
  const int64_t nw = (T + 63) / 64;
  const uint64_t* qw = a.qw + stream * nw;
  const uint64_t* kw = a.kw + stream * nw;
  const uint64_t* vw = a.vw + stream * nw;
  for (int64_t j = threadIdx.x; j < T; j += blockDim.x) sk[j] = window_at(kw, j);
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int64_t nblk = (T + 31) / 32;
  const int64_t b = stream / a.streams, s = stream % a.streams;
  const float pay = a.payload ? a.payload[s] : 1.f;
  // Zig-zag assignment of 32-position blocks keeps the (t-proportional) work balanced.
  for (int64_t round = 0; round * nwarps < nblk; ++round) {
    const int64_t blk = (round & 1) ? ((round + 1) * nwarps - 1 - warp) : (round * nwarps + warp);
    if (blk >= nblk) continue;
    const int64_t t = blk * 32 + lane;
    const bool valid = t < T;
    const uint64_t wq = valid ? window_at(qw, t) : 0ull;
    // longest achievable length at t: min(max_len, t) (j <= t-1 gives L <= t)
    const int cap_t = valid ? (int)min((int64_t)a.max_len, t) : 0;
    int best = 0;
    int64_t bestj = -1;
    // mask of the top (best+1) bits: a key window improves iff they all match
    uint64_t mask = 1ull << 63;
    int64_t j = min(blk * 32 + 31, T - 1) - 1;
    for (; j >= 0; --j) {
      const uint64_t x = wq ^ sk[j];
      if (j < t && best < cap_t && (x & mask) == 0ull && j >= best) {
        int l = x == 0ull ? 64 : __clzll((long long)x);
        const int capj = (int)min((int64_t)cap_t, j + 1);
        l = min(l, capj);
        if (l > best) {
          best = l;
          bestj = j;
          mask = best >= 63 ? ~0ull : ~((~0ull) >> (best + 1));
        }
      }
      if ((j & 31) == 0) {
        // stop when no lane can still find a longer match among j' < j
        const bool can = valid && best < cap_t && (j - 1) >= best;
        if (!__any_sync(0xffffffffu, can)) break;
      }
    }
    if (valid) {
      float sign = -1.f;
      if (bestj >= 0) {
        const int64_t succ = bestj + 1;
        sign = ((vw[succ >> 6] >> (succ & 63)) & 1ull) ? 1.f : -1.f;
      }
      const float o = pay * sign;
      const int64_t off = b * a.ob + t * a.ot + s * a.os;
      if (a.out_dtype == KSD8_F32)
        reinterpret_cast<float*>(a.out)[off] = o;
      else if (a.out_dtype == KSD8_BF16)
        reinterpret_cast<__nv_bfloat16*>(a.out)[off] = __float2bfloat16_rn(o);
      else
        reinterpret_cast<__half*>(a.out)[off] = __float2half_rn(o);
      if (a.match_len) a.match_len[stream * T + t] = best;
      if (a.match_end) a.match_end[stream * T + t] = (int32_t)bestj;
    }
  }
}

// ---------------------------------------------------------------- prefix-table matcher
//
// Same result as rosa_match_kernel in O(1) expected work per position.  One
// warp per stream walks t = 0 .. T-1; before the query at t it inserts key
// position j = t - 1 into 12 tables: level L maps the top L bits of Wk(j) to
// the latest j + 1 with j >= L - 1 (so the padding bits before position 0 never
// count).  The query reads the 12 levels in parallel (lane L - 1 reads level
// L); the highest level that hits is the match length and its entry the latest
// endpoint: a key with a longer effective match would sit in the next level.
// When level 12 hits, the keys sharing those 12 bits are walked newest first
// through per-position links for the exact length (up to the cap); the walk
// stops at the first key reaching min(max_len, t).
#ifndef KSD8_RP_LEVELS
#define KSD8_RP_LEVELS 12
#endif
#ifndef KSD8_RP_WARPS
#define KSD8_RP_WARPS 8
#endif
constexpr int RP_LEVELS = KSD8_RP_LEVELS;      // table levels 1..RP_LEVELS (<= 12)
constexpr int RP_TBL = 1 << (RP_LEVELS + 1);   // level L at offset 2^L - 2
constexpr int RP_WARPS = KSD8_RP_WARPS;        // streams per CTA (fewer when T is long)
constexpr int RP_TMAX = 8192;                  // links are uint16 positions + 1

__device__ __forceinline__ int rp_off(int L) { return (1 << L) - 2; }

// W(t) from words held in shared memory.
__device__ __forceinline__ uint64_t window_sm(const uint64_t* w, int64_t t) {
  const int64_t wi = t >> 6;
  const int sh = (int)(t & 63) + 1;
  const uint64_t hi = w[wi];
  const uint64_t lo = wi > 0 ? w[wi - 1] : 0ull;
  return sh == 64 ? hi : ((lo >> sh) | (hi << (64 - sh)));
}

// Per-warp shared memory: level tables (RP_TBL uint16), chain links (T
// uint16), then the stream's q, k and v bit words (3 x ceil(T/64) uint64).
__global__ void __launch_bounds__(RP_WARPS * 32) rosa_match_prefix_kernel(MatchArgs a,
                                                                           int stride) {
  extern __shared__ __align__(16) uint8_t rsm_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stream = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (stream >= a.batch * a.streams) return;  // the whole warp: no CTA barrier below
  const int64_t T = a.t_len;
  const int64_t nw = (T + 63) / 64;
  uint8_t* base = rsm_raw + (size_t)warp * stride;
  uint16_t* tbl = reinterpret_cast<uint16_t*>(base);
  uint16_t* prev = tbl + RP_TBL;
  uint64_t* sq = reinterpret_cast<uint64_t*>(base + (((size_t)RP_TBL + T) * 2 + 15) / 16 * 16);
  uint64_t* sk = sq + nw;
  uint64_t* sv = sk + nw;
  for (int i = lane; i < RP_TBL / 8; i += 32) reinterpret_cast<uint4*>(tbl)[i] = make_uint4(0, 0, 0, 0);
  for (int64_t i = lane; i < nw; i += 32) {
    sq[i] = a.qw[stream * nw + i];
    sk[i] = a.kw[stream * nw + i];
    sv[i] = a.vw[stream * nw + i];
  }
  __syncwarp();
  const int64_t b = stream / a.streams, s = stream % a.streams;
  const float pay = a.payload ? a.payload[s] : 1.f;
  const int L = lane + 1;               // this lane's level (lanes 0..11)
  const int off = lane < RP_LEVELS ? rp_off(L) : 0;
  for (int64_t t = 0; t < T; ++t) {
    // insert key position j = t - 1 into this lane's level; the query below
    // reads the same level from the same lane, so no barrier is needed
    if (t >= 1 && lane < RP_LEVELS && t >= L) {
      const int64_t j = t - 1;
      const int idx = off + (int)(window_sm(sk, j) >> (64 - L));
      if (L == RP_LEVELS) prev[j] = tbl[idx];
      tbl[idx] = (uint16_t)t;             // j + 1
    }
    const uint64_t wq = window_sm(sq, t);
    const int cap = (int)min((int64_t)a.max_len, t);
    uint32_t hj = 0;
    if (lane < RP_LEVELS && L <= cap) hj = tbl[off + (int)(wq >> (64 - L))];
    const unsigned mask = __ballot_sync(0xffffffffu, hj != 0);
    int best = 0;
    int64_t bestj = -1;
    if (mask) {
      const int lh = 32 - __clz((int)mask);
      const uint32_t head = __shfl_sync(0xffffffffu, hj, lh - 1);
      best = lh;
      bestj = (int64_t)head - 1;
      if (lh == RP_LEVELS && cap > RP_LEVELS) {
        __syncwarp();  // the chain links were written by the level-12 lane
        best = 0;
        bestj = -1;
        for (uint32_t c = head; c != 0;) {
          const int64_t j = (int64_t)c - 1;
          const uint64_t x = wq ^ window_sm(sk, j);
          int l = x == 0ull ? 64 : __clzll((long long)x);
          l = min(l, (int)min((int64_t)cap, j + 1));
          if (l > best) {
            best = l;
            bestj = j;
            if (best == cap) break;
          }
          c = prev[j];
        }
      }
    }
    if (lane == (int)(t & 31)) {
      float sign = -1.f;
      if (bestj >= 0) {
        const int64_t succ = bestj + 1;
        sign = ((sv[succ >> 6] >> (succ & 63)) & 1ull) ? 1.f : -1.f;
      }
      const float o = pay * sign;
      const int64_t oo = b * a.ob + t * a.ot + s * a.os;
      if (a.out_dtype == KSD8_F32)
        reinterpret_cast<float*>(a.out)[oo] = o;
      else if (a.out_dtype == KSD8_BF16)
        reinterpret_cast<__nv_bfloat16*>(a.out)[oo] = __float2bfloat16_rn(o);
      else
        reinterpret_cast<__half*>(a.out)[oo] = __float2half_rn(o);
      if (a.match_len) a.match_len[stream * T + t] = best;
      if (a.match_end) a.match_end[stream * T + t] = (int32_t)bestj;
    }
  }
}

// Keys of one k word (mask M) whose windows agree with wq in the top bits:
// the longest such agreement (<= cap) and, in mout, the keys reaching it.
// first_word: word 0, where a key j is also capped at j + 1.
__device__ __forceinline__ int bits_word_match(uint64_t kwd, uint64_t kprev, uint64_t M,
                                               uint64_t wq, int cap, bool first_word,
                                               uint64_t& mout) {
  int len = 0;
  while (len < cap) {
    const uint64_t sh = len ? ((kwd << len) | (kprev >> (64 - len))) : kwd;
    uint64_t e = ((wq >> (63 - len)) & 1ull) ? sh : ~sh;
    if (first_word) e &= ~0ull << len;  // length <= j + 1
    const uint64_t m2 = M & e;
    if (!m2) break;
    M = m2;
    ++len;
  }
  mout = M;
  return len;
}

// ---------------------------------------------------------------- chunked matcher
//
// The same prefix tables, processed 32 positions at a time: lane i owns query
// t = t0 + i and key j = t0 - 1 + i.  The tables hold the keys j <= t0 - 2
// (inserted by earlier chunks); each lane reads its query's 12 levels itself
// (independent loads) and walks the level-12 chain when it hits; the keys of
// the chunk itself (t0 - 1 <= j <= t - 1) are compared directly, broadcast by
// shuffles.  A longest match found among the chunk's keys is later than any
// table key, so it wins ties.  Then the chunk's 32 keys are inserted into
// every level at once: lanes whose prefixes collide are grouped with
// match_any, the highest lane (latest key) writes the level entry, and the
// level-12 links point each key at the next older key of its group (or at the
// previous head).  About 12 warp instructions per position instead of ~175
// for the one-position-per-step walk, with 12 independent table loads per
// lane instead of a dependent chain.  The chunk's own keys are matched
// bit-parallel over their k words (bits_word_match), and past the first chunk
// the 12 levels' groupings are formed together before one round of writes.
// Config-4 layer, fair bits: 2.28 ms -> 1.97 (batched insertion) -> 1.48 ms.
#ifndef KSD8_RC_WARPS
#define KSD8_RC_WARPS 16
#endif
constexpr int RC_WARPS = KSD8_RC_WARPS;  // streams per CTA, up to what shared memory holds

__global__ void __launch_bounds__(RC_WARPS * 32) rosa_match_chunk_kernel(MatchArgs a,
                                                                          int stride) {
  extern __shared__ __align__(16) uint8_t rsm_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t stream = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (stream >= a.batch * a.streams) return;  // the whole warp: no CTA barrier below
  const int64_t T = a.t_len;
  const int64_t nw = (T + 63) / 64;
  uint8_t* base = rsm_raw + (size_t)warp * stride;
  uint16_t* tbl = reinterpret_cast<uint16_t*>(base);
  uint16_t* prev = tbl + RP_TBL;
  uint64_t* sq = reinterpret_cast<uint64_t*>(base + (((size_t)RP_TBL + T) * 2 + 15) / 16 * 16);
  uint64_t* sk = sq + nw;
  uint64_t* sv = sk + nw;
  for (int i = lane; i < RP_TBL / 8; i += 32) reinterpret_cast<uint4*>(tbl)[i] = make_uint4(0, 0, 0, 0);
  for (int64_t i = lane; i < nw; i += 32) {
    sq[i] = a.qw[stream * nw + i];
    sk[i] = a.kw[stream * nw + i];
    sv[i] = a.vw[stream * nw + i];
  }
  __syncwarp();
  const int64_t b = stream / a.streams, s = stream % a.streams;
  const float pay = a.payload ? a.payload[s] : 1.f;
  const unsigned full = 0xffffffffu;
  uint64_t walked = 0;   // chain steps of this stream so far (warp total)
  for (int64_t t0 = 0; t0 < T; t0 += 32) {
    const int64_t t = t0 + lane;
    const bool valid = t < T;
    const uint64_t wq = valid ? window_sm(sq, t) : 0ull;
    const int cap = valid ? (int)min((int64_t)a.max_len, t) : 0;
    const int64_t jk = t0 - 1 + lane;                  // this lane's key
    const bool kin = jk >= 0 && jk < T;
    const uint64_t wk = kin ? window_sm(sk, jk) : 0ull;

    // keys of earlier chunks: the highest level whose L-bit prefix is present
    uint32_t hit[RP_LEVELS];
#pragma unroll
    for (int L = 1; L <= RP_LEVELS; ++L)
      hit[L - 1] = L <= cap ? tbl[rp_off(L) + (int)(wq >> (64 - L))] : 0u;
    int best = 0;
    int64_t bestj = -1;
#pragma unroll
    for (int L = 1; L <= RP_LEVELS; ++L)
      if (hit[L - 1]) {
        best = L;
        bestj = (int64_t)hit[L - 1] - 1;
      }
    int steps = 0;
    if (best == RP_LEVELS && cap > RP_LEVELS) {
      // exact length among the keys sharing the top RP_LEVELS bits, newest first
      const uint32_t head = hit[RP_LEVELS - 1];
      best = 0;
      bestj = -1;
      for (uint32_t c = head; c != 0; ++steps) {
        const int64_t j = (int64_t)c - 1;
        const uint64_t x = wq ^ window_sm(sk, j);
        int l = x == 0ull ? 64 : __clzll((long long)x);
        l = min(l, (int)min((int64_t)cap, j + 1));
        if (l > best) {
          best = l;
          bestj = j;
          if (best == cap) break;
        }
        c = prev[j];
      }
    }
    // keys of this chunk, j = t0 - 1 .. t - 1, bit-parallel over their (at most
    // two) k words, the later word first
    int lc = 0;
    int64_t jc = -1;
    if (cap > 0) {
      const int64_t jlo = t0 > 0 ? t0 - 1 : 0, jhi = t - 1;
      for (int64_t w = jhi >> 6; w >= (jlo >> 6) && jhi >= jlo; --w) {
        const int lo_b = (int)max(jlo - (w << 6), (int64_t)0);
        const int hi_b = (int)min(jhi - (w << 6), (int64_t)63);
        const uint64_t M = (~0ull << lo_b) & (~0ull >> (63 - hi_b));
        uint64_t mo;
        const int l = bits_word_match(sk[w], w > 0 ? sk[w - 1] : 0ull, M, wq, cap, w == 0, mo);
        if (l > lc) {
          lc = l;
          jc = (w << 6) + 63 - __clzll((long long)mo);
        }
      }
    }
    if (lc > 0 && lc >= best) {
      best = lc;
      bestj = jc;
    }
    if (valid) {
      float sign = -1.f;
      if (bestj >= 0) {
        const int64_t succ = bestj + 1;
        sign = ((sv[succ >> 6] >> (succ & 63)) & 1ull) ? 1.f : -1.f;
      }
      const float o = pay * sign;
      const int64_t oo = b * a.ob + t * a.ot + s * a.os;
      if (a.out_dtype == KSD8_F32)
        reinterpret_cast<float*>(a.out)[oo] = o;
      else if (a.out_dtype == KSD8_BF16)
        reinterpret_cast<__nv_bfloat16*>(a.out)[oo] = __float2bfloat16_rn(o);
      else
        reinterpret_cast<__half*>(a.out)[oo] = __float2half_rn(o);
      if (a.match_len) a.match_len[stream * T + t] = best;
      if (a.match_end) a.match_end[stream * T + t] = (int32_t)bestj;
    }

    // insert this chunk's keys: level L takes key j when j >= L - 1
    __syncwarp();  // every lane has finished reading the tables of this chunk
    if (t0 >= RP_LEVELS) {
      // every key of the chunk enters every level: the 12 groupings are
      // independent, so they are formed together, the old level-12 heads read,
      // and then all entries written (one warp barrier instead of one per level)
      const unsigned im = __ballot_sync(full, kin);
      if (kin) {
        unsigned grp[RP_LEVELS];
#pragma unroll
        for (int L = 1; L <= RP_LEVELS; ++L)
          grp[L - 1] = __match_any_sync(im, rp_off(L) + (int)(wk >> (64 - L)));
        const int idx12 = rp_off(RP_LEVELS) + (int)(wk >> (64 - RP_LEVELS));
        const unsigned lower = grp[RP_LEVELS - 1] & ((1u << lane) - 1u);
        prev[jk] = lower ? (uint16_t)(t0 + (31 - __clz((int)lower))) : tbl[idx12];
        __syncwarp(im);  // the old heads are read before the newest keys replace them
#pragma unroll
        for (int L = 1; L <= RP_LEVELS; ++L)
          if (lane == 31 - __clz((int)grp[L - 1]))
            tbl[rp_off(L) + (int)(wk >> (64 - L))] = (uint16_t)(jk + 1);
      }
      __syncwarp();
    } else
#pragma unroll
    for (int L = 1; L <= RP_LEVELS; ++L) {
      const bool ins = kin && jk >= L - 1;
      const unsigned im = __ballot_sync(full, ins);
      if (ins) {
        const int idx = rp_off(L) + (int)(wk >> (64 - L));
        const unsigned grp = __match_any_sync(im, idx);
        if (L == RP_LEVELS) {
          const unsigned lower = grp & ((1u << lane) - 1u);
          prev[jk] = lower ? (uint16_t)(t0 + (31 - __clz((int)lower)))  // (t0-1+i) + 1
                           : tbl[idx];
        }
        __syncwarp(im);  // the old head is read before the newest key replaces it
        if (lane == 31 - __clz((int)grp)) tbl[idx] = (uint16_t)(jk + 1);
      }
      __syncwarp();
    }
    if (a.redo) {
      // long runs make the chains long (O(T) per position): leave such a stream to
      // the sorted matcher, which rewrites all of its positions
      walked += __reduce_add_sync(full, (unsigned)steps);
      if (t0 >= 96 && walked > (uint64_t)a.redo_budget * (uint64_t)(t0 + 32)) {
        if (lane == 0) {
          const int slot = atomicAdd(a.redo, 1);
          a.redo[1 + slot] = (int32_t)stream;
        }
        return;
      }
    }
  }
}

// ---------------------------------------------------------------- sorted-key matcher
//
// Exact, with O(log T) work per position whatever the bit statistics (the
// level-12 chains of the prefix tables degenerate to O(T) walks on streams with
// long runs, as the projections of trained or deep-layer activations give).
//
// The 64-bit window W(j) of a key determines its common-suffix length with a
// query window: lcs = clz(Wq(t) ^ Wk(j)).  With the keys j >= R0 = max_len - 1
// (whose window has at least max_len real bits) sorted by window value, the
// keys sharing the top L bits with a query form one interval of ranks, and the
// largest common prefix with any inserted key is reached at the inserted
// predecessor or successor of the query's rank.  Per stream (one warp):
//   - bitonic sort of the (window, j) pairs of the keys j in [R0, T-2];
//   - 32 queries per step (lane = t0 + lane), against the keys inserted so far
//     (j <= t0 - 2): binary search of the rank, inserted neighbours from a
//     bitmap with a summary word, L = min(max lcp, cap_t), the rank interval of
//     the L-bit prefix by two binary searches, and the latest endpoint in it
//     from a max segment tree over ranks;
//   - keys j < R0 (their window reaches before position 0, so a match is also
//     capped at j + 1) and this step's own keys j in [t0-1, t-1] are compared
//     directly (broadcast loads / shuffles);
//   - then this step's keys are inserted (bitmap bits, segment-tree maxima;
//     keys sharing a tree node are grouped with match_any and the latest wins).
constexpr int RS_MAXNP = 4096;  // sorted keys per stream (T <= 4096 + R0)

__device__ __forceinline__ bool rs_less(uint64_t wa, uint16_t ja, uint64_t wb, uint16_t jb) {
  return wa < wb || (wa == wb && ja < jb);
}

// number of sorted windows < key (first rank with SW[rank] >= key); np a power of 2
__device__ __forceinline__ int rs_lower_bound(const uint64_t* sw, int np, uint64_t key) {
  int pos = 0;
  for (int step = np >> 1; step > 0; step >>= 1)
    if (sw[pos + step - 1] < key) pos += step;
  return (pos == np - 1 && sw[pos] < key) ? np : pos;
}

// rs_lower_bound of two keys at once: the two searches are independent, so
// their shared-memory loads overlap
__device__ __forceinline__ void rs_lower_bound2(const uint64_t* sw, int np, uint64_t k1,
                                                uint64_t k2, int& r1, int& r2) {
  int p1 = 0, p2 = 0;
  for (int step = np >> 1; step > 0; step >>= 1) {
    const uint64_t a = sw[p1 + step - 1], b = sw[p2 + step - 1];
    if (a < k1) p1 += step;
    if (b < k2) p2 += step;
  }
  r1 = (p1 == np - 1 && sw[p1] < k1) ? np : p1;
  r2 = (p2 == np - 1 && sw[p2] < k2) ? np : p2;
}

// largest inserted rank < r (-1 if none); bitmap words bm (32 bits), summary sm[2]
__device__ __forceinline__ int rs_pred(const uint32_t* bm, const uint64_t* sm, int r) {
  if (r <= 0) return -1;
  const int q = r - 1;
  const int w = q >> 5;
  const uint32_t m = bm[w] & (0xFFFFFFFFu >> (31 - (q & 31)));
  if (m) return (w << 5) + 31 - __clz((int)m);
  for (int h = w >> 6; h >= 0; --h) {
    uint64_t sw = sm[h];
    if (h == (w >> 6)) sw &= (w & 63) ? (~0ull >> (64 - (w & 63))) : 0ull;
    if (sw) {
      const int w2 = (h << 6) + 63 - __clzll((long long)sw);
      return (w2 << 5) + 31 - __clz((int)bm[w2]);
    }
  }
  return -1;
}

// smallest inserted rank >= r (-1 if none), ranks < np
__device__ __forceinline__ int rs_succ(const uint32_t* bm, const uint64_t* sm, int r, int np) {
  if (r >= np) return -1;
  const int w = r >> 5;
  const uint32_t m = bm[w] & (0xFFFFFFFFu << (r & 31));
  if (m) return (w << 5) + __ffs((int)m) - 1;
  const int nwords = np >> 5;
  for (int h = w >> 6; (h << 6) < nwords; ++h) {
    uint64_t sw = sm[h];
    if (h == (w >> 6)) sw &= ((w & 63) == 63) ? 0ull : (~0ull << ((w & 63) + 1));
    if (sw) {
      const int w2 = (h << 6) + __ffsll((long long)sw) - 1;
      return (w2 << 5) + __ffs((int)bm[w2]) - 1;
    }
  }
  return -1;
}

__global__ void __launch_bounds__(RC_WARPS * 32) rosa_match_sorted_kernel(MatchArgs a, int np,
                                                                           int stride) {
  extern __shared__ __align__(16) uint8_t rsm_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t stream = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (a.redo_pass) {  // only the streams the chunked kernel handed over
    if (stream >= a.redo[0]) return;
    stream = a.redo[1 + stream];
  }
  if (stream >= a.batch * a.streams) return;  // the whole warp: no CTA barrier below
  const int T = (int)a.t_len;
  const int nw = (T + 63) / 64;
  const int ml = a.max_len;
  const int r0 = ml > 0 ? ml - 1 : 0;        // first key whose window has max_len real bits
  const int nk = T - 1 - r0 > 0 ? T - 1 - r0 : 0;  // sorted keys j in [r0, T-2]
  // per-warp layout: SW[np] u64 | seg[2np] u16 (holds SJ[np] while sorting) |
  //                  rank_of[T] u16 | bm[np/32] u32 | sm[2] u64 | sq, sk, sv [nw] u64
  uint8_t* base = rsm_raw + (size_t)warp * stride;
  uint64_t* SW = reinterpret_cast<uint64_t*>(base);
  uint16_t* seg = reinterpret_cast<uint16_t*>(SW + np);
  uint16_t* SJ = seg;
  uint16_t* rank_of = seg + 2 * np;
  uint32_t* bm = reinterpret_cast<uint32_t*>(
      base + (((size_t)np * 8 + (size_t)4 * np + (size_t)2 * T + 15) / 16 * 16));
  uint64_t* sm = reinterpret_cast<uint64_t*>(bm + np / 32);
  uint64_t* sq = sm + 2;
  uint64_t* sk = sq + nw;
  uint64_t* sv = sk + nw;
  uint64_t* EW = sv + nw;   // windows of the keys j < r0 (at most 64)
  for (int i = lane; i < nw; i += 32) {
    sq[i] = a.qw[stream * nw + i];
    sk[i] = a.kw[stream * nw + i];
    sv[i] = a.vw[stream * nw + i];
  }
  for (int i = lane; i < np / 32; i += 32) bm[i] = 0u;
  if (lane < 2) sm[lane] = 0ull;
  __syncwarp();
  for (int i = lane; i < r0 && i < T; i += 32) EW[i] = window_sm(sk, i);
  for (int i = lane; i < np; i += 32) {
    const bool real = i < nk;
    SW[i] = real ? window_sm(sk, r0 + i) : ~0ull;
    SJ[i] = real ? (uint16_t)(r0 + i) : (uint16_t)0xFFFFu;
  }
  __syncwarp();
  // bitonic sort of (SW, SJ) ascending; each lane takes compare-exchange pairs
  // (i, i + jj), i with bit jj clear, so no lane idles on the upper halves
  for (int k = 2; k <= np; k <<= 1) {
    for (int jj = k >> 1; jj > 0; jj >>= 1) {
      for (int pr = lane; pr < (np >> 1); pr += 32) {
        const int i = ((pr & ~(jj - 1)) << 1) | (pr & (jj - 1));
        const int l = i | jj;
        const bool up = (i & k) == 0;
        const uint64_t wi = SW[i], wl = SW[l];
        const uint16_t ji = SJ[i], jl = SJ[l];
        if (rs_less(wl, jl, wi, ji) == up) {
          SW[i] = wl; SW[l] = wi;
          SJ[i] = jl; SJ[l] = ji;
        }
      }
      __syncwarp();
    }
  }
  for (int i = lane; i < nk; i += 32) rank_of[SJ[i]] = (uint16_t)i;
  __syncwarp();
  for (int i = lane; i < 2 * np; i += 32) seg[i] = 0;   // SJ is spent: the tree starts empty
  __syncwarp();

  const int64_t b = stream / a.streams, s = stream % a.streams;
  const float pay = a.payload ? a.payload[s] : 1.f;
  const unsigned full = 0xffffffffu;
  for (int t0 = 0; t0 < T; t0 += 32) {
    const int t = t0 + lane;
    const bool valid = t < T;
    const uint64_t wq = valid ? window_sm(sq, t) : 0ull;
    const int cap = valid ? min(ml, t) : 0;
    const int jk = t0 - 1 + lane;                       // this lane's key
    const bool kin = jk >= 0 && jk < T;
    const uint64_t wk = kin ? window_sm(sk, jk) : 0ull;
    int best = 0, bestj = -1;
    // sorted keys inserted by earlier steps (r0 <= j <= t0 - 2)
    if (t0 - 2 >= r0 && cap > 0) {
      const int r = rs_lower_bound(SW, np, wq);
      const int p = rs_pred(bm, sm, r), q = rs_succ(bm, sm, r, np);
      int lraw = 0;
      if (p >= 0) { const uint64_t x = wq ^ SW[p]; lraw = x ? __clzll((long long)x) : 64; }
      if (q >= 0) { const uint64_t x = wq ^ SW[q]; lraw = max(lraw, x ? __clzll((long long)x) : 64); }
      const int L = min(lraw, cap);
      if (L > 0) {
        const uint64_t pre = L >= 64 ? wq : (wq >> (64 - L)) << (64 - L);
        const uint64_t last = L >= 64 ? wq : pre | (~0ull >> L);
        int lo, hi;   // [lo, hi): the ranks sharing the top L bits
        rs_lower_bound2(SW, np, pre, last == ~0ull ? last : last + 1, lo, hi);
        if (last == ~0ull) hi = np;
        int res = 0;
        for (int l = lo + np, h = hi + np; l < h; l >>= 1, h >>= 1) {
          if (l & 1) res = max(res, (int)seg[l++]);
          if (h & 1) res = max(res, (int)seg[--h]);
        }
        best = L;
        bestj = res - 1;
      }
    }
    // keys j < r0: also capped at j + 1; only those with j >= best can improve
    {
      const int jhi = min(r0 - 1, t0 - 2);
      int jlo = valid ? best : 0x7fffffff;
      jlo = __reduce_min_sync(full, jlo);
      // candidates packed as (length << 8) | j, four independent running maxima
      int pk[4] = {0, 0, 0, 0};
      int j = jlo;
      for (; j + 3 <= jhi; j += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint64_t x = wq ^ EW[j + u];
          int l = x ? __clzll((long long)x) : 64;
          l = min(l, min(cap, j + u + 1));
          pk[u] = max(pk[u], l > 0 ? ((l << 8) | (j + u)) : 0);
        }
      }
      for (; j <= jhi; ++j) {
        const uint64_t x = wq ^ EW[j];
        int l = x ? __clzll((long long)x) : 64;
        l = min(l, min(cap, j + 1));
        pk[0] = max(pk[0], l > 0 ? ((l << 8) | j) : 0);
      }
      const int top = max(max(pk[0], pk[1]), max(pk[2], pk[3]));
      if ((top >> 8) > best) { best = top >> 8; bestj = top & 0xFF; }
    }
    // this step's own keys, j = t0 - 1 + i <= t - 1 (the latest: they win ties):
    // candidates packed as (length << 8) | i, four independent running maxima
    {
      int pk[4] = {0, 0, 0, 0};
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint64_t wki = __shfl_sync(full, wk, i);
        const int j = t0 - 1 + i;
        const uint64_t x = wq ^ wki;
        int l = x ? __clzll((long long)x) : 64;
        l = min(l, min(cap, j + 1));
        const int c = (i <= lane && j >= 0 && l > 0) ? ((l << 8) | i) : 0;
        pk[i & 3] = max(pk[i & 3], c);
      }
      const int top = max(max(pk[0], pk[1]), max(pk[2], pk[3]));
      if (top && (top >> 8) >= best) {
        best = top >> 8;
        bestj = t0 - 1 + (top & 0xFF);
      }
    }
    if (valid) {
      float sign = -1.f;
      if (bestj >= 0) {
        const int succ = bestj + 1;
        sign = ((sv[succ >> 6] >> (succ & 63)) & 1ull) ? 1.f : -1.f;
      }
      const float o = pay * sign;
      const int64_t oo = b * a.ob + (int64_t)t * a.ot + s * a.os;
      if (a.out_dtype == KSD8_F32)
        reinterpret_cast<float*>(a.out)[oo] = o;
      else if (a.out_dtype == KSD8_BF16)
        reinterpret_cast<__nv_bfloat16*>(a.out)[oo] = __float2bfloat16_rn(o);
      else
        reinterpret_cast<__half*>(a.out)[oo] = __float2half_rn(o);
      if (a.match_len) a.match_len[stream * a.t_len + t] = best;
      if (a.match_end) a.match_end[stream * a.t_len + t] = bestj;
    }
    // insert this step's sorted keys (r0 <= j <= T - 2)
    __syncwarp();
    const bool ins = kin && jk >= r0 && jk <= T - 2;
    const unsigned im = __ballot_sync(full, ins);
    if (ins) {
      const int r = rank_of[jk];
      atomicOr(&bm[r >> 5], 1u << (r & 31));
      atomicOr((unsigned long long*)&sm[r >> 11], 1ull << ((r >> 5) & 63));
      for (int node = r + np; node >= 1; node >>= 1) {
        const unsigned grp = __match_any_sync(im, node);
        if (lane == 31 - __clz((int)grp)) seg[node] = (uint16_t)(jk + 1);
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------- bit-parallel matcher
//
// Exact, O(T / 64 x matched bits) per position and no per-stream index: for
// query t, the keys of one k word (64 consecutive positions j) whose windows
// agree with Wq(t) in the top l bits form a bit mask M_l = M_{l-1} & E_l,
// where E_l marks k[j - l] == q[t - l] (the k word shifted up by l, the bits
// below position 0 reading 0).  The loop narrows M until it empties or
// reaches the cap: the surviving keys all have that length, the highest bit
// is the latest of them.  Words are taken latest first, so an earlier word
// only replaces a strictly longer match; the search stops at the cap.  In
// word 0 a key j is also capped at j + 1 (E_l keeps only j >= l).  One warp
// per stream, lane = query, 3 x ceil(T / 64) words of shared memory per warp.
__global__ void __launch_bounds__(256) rosa_match_bits_kernel(MatchArgs a) {
  extern __shared__ __align__(16) uint64_t rbw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t stream = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  if (a.redo_pass) {  // only the streams the chunked kernel handed over
    if (stream >= a.redo[0]) return;
    stream = a.redo[1 + stream];
  }
  if (stream >= a.batch * a.streams) return;  // the whole warp: no CTA barrier below
  const int64_t T = a.t_len;
  const int nw = (int)((T + 63) / 64);
  const int ml = a.max_len;
  uint64_t* sq = rbw + (size_t)warp * 3 * nw;
  uint64_t* sk = sq + nw;
  uint64_t* sv = sk + nw;
  for (int i = lane; i < nw; i += 32) {
    sq[i] = a.qw[stream * nw + i];
    sk[i] = a.kw[stream * nw + i];
    sv[i] = a.vw[stream * nw + i];
  }
  __syncwarp();
  const int64_t b = stream / a.streams, s = stream % a.streams;
  const float pay = a.payload ? a.payload[s] : 1.f;
  for (int64_t t0 = 0; t0 < T; t0 += 32) {
    const int64_t t = t0 + lane;
    if (t >= T) break;
    const uint64_t wq = window_sm(sq, t);
    const int cap = (int)min((int64_t)ml, t);
    int best = 0;
    int64_t bestj = -1;
    if (cap > 0) {
      // keys j <= t - 1, word by word from the latest
      const int64_t wl = (t - 1) >> 6;
      uint64_t M = ~0ull >> (63 - (int)((t - 1) & 63));   // j <= t - 1 in the latest word
      for (int64_t w = wl; w >= 1; --w) {
        uint64_t mo;
        const int len = bits_word_match(sk[w], sk[w - 1], M, wq, cap, false, mo);
        if (len > best) {
          best = len;
          bestj = (w << 6) + 63 - __clzll((long long)mo);
          if (best == cap) break;
        }
        M = ~0ull;
      }
      if (best < cap) {
        uint64_t mo;
        const int len = bits_word_match(sk[0], 0ull, wl == 0 ? M : ~0ull, wq, cap, true, mo);
        if (len > best) {
          best = len;
          bestj = 63 - __clzll((long long)mo);
        }
      }
    }
    float sign = -1.f;
    if (bestj >= 0) {
      const int64_t succ = bestj + 1;
      sign = ((sv[succ >> 6] >> (succ & 63)) & 1ull) ? 1.f : -1.f;
    }
    const float o = pay * sign;
    const int64_t oo = b * a.ob + t * a.ot + s * a.os;
    if (a.out_dtype == KSD8_F32)
      reinterpret_cast<float*>(a.out)[oo] = o;
    else if (a.out_dtype == KSD8_BF16)
      reinterpret_cast<__nv_bfloat16*>(a.out)[oo] = __float2bfloat16_rn(o);
    else
      reinterpret_cast<__half*>(a.out)[oo] = __float2half_rn(o);
    if (a.match_len) a.match_len[stream * a.t_len + t] = best;
    if (a.match_end) a.match_end[stream * a.t_len + t] = (int32_t)bestj;
  }
}

struct TimemixArgs {
  const void* x;
  int64_t batch, t_len, d;
  const float* mix[3];
  int8_t* codes[3];
  __half* scales[3];
};

// One warp per (128-wide group, run of TM_TOKENS consecutive tokens); a lane
// owns 4 consecutive features.  The mix factors stay in registers for the
// run, a token's row is the next token's `prev` (one load per element), and
// the codes come from the packed four-code path (gs_code4_normal: one
// multiply by RN(1/scale) and the 1.5 * 2^23 shifter, the IEEE division only
// near a rounding tie), as in the row quantiser.
constexpr int TM_TOKENS = 16;

template <typename T>
__device__ __forceinline__ void load4f(const T* p, bool full, int n, float (&o)[4]) {
  if constexpr (sizeof(T) == 4) {
    if (full) {
      const float4 v = *reinterpret_cast<const float4*>(p);
      o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
      return;
    }
  } else {
    if (full) {
      const uint2 v = *reinterpret_cast<const uint2*>(p);
      const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = (float)h[i];
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = i < n ? (float)p[i] : 0.f;
}

template <typename T>
__global__ void __launch_bounds__(256) rosa_timemix_quant_kernel(TimemixArgs a) {
  const int64_t groups = (a.d + 127) / 128;
  const int64_t tokens = a.batch * a.t_len;
  const int64_t runs = (tokens + TM_TOKENS - 1) / TM_TOKENS;
  const int64_t total = groups * runs;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const T* x = reinterpret_cast<const T*>(a.x);
  // vector loads need 4 whole features in range and 16-/8-byte aligned rows
  const bool vec = (a.d % 4) == 0 && (reinterpret_cast<uintptr_t>(a.x) % (4 * sizeof(T))) == 0;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total;
       w += nwarps) {
    const int64_t g = w % groups, run = w / groups;
    const int64_t c = g * 128 + lane * 4;
    const int n = (int)max((int64_t)0, min((int64_t)4, a.d - c));
    const bool full = vec && n == 4;
    float mix[3][4];
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
      for (int i = 0; i < 4; ++i) mix[p][i] = i < n ? a.mix[p][c + i] : 0.f;
    const int64_t tok0 = run * TM_TOKENS;
    const int64_t tok1 = min(tokens, tok0 + TM_TOKENS);
    float prev[4] = {0.f, 0.f, 0.f, 0.f};
    if (tok0 % a.t_len != 0 && n > 0) load4f(x + (tok0 - 1) * a.d + c, full, n, prev);
    for (int64_t tok = tok0; tok < tok1; ++tok) {
      if (tok % a.t_len == 0) {  // a sequence starts: prev is the zero padding
#pragma unroll
        for (int i = 0; i < 4; ++i) prev[i] = 0.f;
      }
      float cur[4] = {0.f, 0.f, 0.f, 0.f};
      if (n > 0) load4f(x + tok * a.d + c, full, n, cur);
      float diff[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // (x - prev) is evaluated in x's dtype
        if constexpr (sizeof(T) == 2) diff[i] = (float)(T)(cur[i] - prev[i]);
        else diff[i] = cur[i] - prev[i];
      }
      // the three projection inputs, their group maxima reduced together
      float vv[3][4], mm[3];
#pragma unroll
      for (int p = 0; p < 3; ++p) {
#pragma unroll
        for (int i = 0; i < 4; ++i) vv[p][i] = __fadd_rn(prev[i], __fmul_rn(diff[i], mix[p][i]));
        mm[p] = fmaxf(fmaxf(fabsf(vv[p][0]), fabsf(vv[p][1])), fmaxf(fabsf(vv[p][2]), fabsf(vv[p][3])));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int p = 0; p < 3; ++p) mm[p] = fmaxf(mm[p], __shfl_xor_sync(0xffffffffu, mm[p], o));
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const float (&v)[4] = vv[p];
        const float m = mm[p];
        __half sh;
        const float scale = gs_scale_fast(m, &sh);
        int8_t* out = a.codes[p] + tok * a.d + c;
        if (n == 4 && gs_scale_is_normal(m, scale) && (reinterpret_cast<uintptr_t>(out) & 3) == 0) {
          *reinterpret_cast<uint32_t*>(out) = gs_code4_normal(v, scale, rcp_approx(scale));
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (i < n) out[i] = (int8_t)gs_code(v[i], scale);
        }
        if (lane == 0) a.scales[p][tok * groups + g] = sh;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) prev[i] = cur[i];
    }
  }
}

__global__ void adamw_kernel(float* p, const void* g, int gdt, float* m, float* v, int64_t n,
                             float lr, float b1, float b2, float eps, float wd, float bc1,
                             float bc2_sqrt, const float* gscale) {
  // gradient clipping (torch.nn.utils.clip_grad_norm_): grads *= coefficient,
  // read from device memory so that no host round trip decides it
  const float gs = gscale ? *gscale : 1.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float gr = gdt == KSD8_F16 ? __half2float(reinterpret_cast<const __half*>(g)[i])
               : gdt == KSD8_BF16
                   ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g)[i])
                   : reinterpret_cast<const float*>(g)[i];
    if (gscale) gr = __fmul_rn(gr, gs);
    float pi = p[i] * (1.f - lr * wd);
    const float mi = b1 * m[i] + (1.f - b1) * gr;
    const float vi = b2 * v[i] + (1.f - b2) * gr * gr;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    pi -= (lr / bc1) * mi / denom;
    p[i] = pi;
  }
}

// AdamW over up to KSD8_ADAMW_MULTI tensors in one launch (same arithmetic as
// adamw_kernel); every thread walks the tensors in order.
struct AdamwMulti {
  float* p[KSD8_ADAMW_MULTI];
  const void* g[KSD8_ADAMW_MULTI];
  float* m[KSD8_ADAMW_MULTI];
  float* v[KSD8_ADAMW_MULTI];
  int64_t n[KSD8_ADAMW_MULTI];
  int count;
};

__global__ void adamw_multi_kernel(AdamwMulti t, int gdt, float lr, float b1, float b2, float eps,
                                   float wd, float bc1, float bc2_sqrt, const float* gscale) {
  const float gs = gscale ? *gscale : 1.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int k = 0; k < t.count; ++k) {
    float* p = t.p[k];
    float* m = t.m[k];
    float* v = t.v[k];
    const void* g = t.g[k];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < t.n[k]; i += stride) {
      float gr = gdt == KSD8_F16 ? __half2float(reinterpret_cast<const __half*>(g)[i])
                 : gdt == KSD8_BF16
                     ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g)[i])
                     : reinterpret_cast<const float*>(g)[i];
      if (gscale) gr = __fmul_rn(gr, gs);
      float pi = p[i] * (1.f - lr * wd);
      const float mi = b1 * m[i] + (1.f - b1) * gr;
      const float vi = b2 * v[i] + (1.f - b2) * gr * gr;
      m[i] = mi;
      v[i] = vi;
      const float denom = sqrtf(vi) / bc2_sqrt + eps;
      pi -= (lr / bc1) * mi / denom;
      p[i] = pi;
    }
  }
}

// Sum of squares of n fp32 values: per-block partial sums (fixed tree order)
// into partials[blockIdx.x].
constexpr int GN_BLOCKS = 592;  // 4 x 148
__global__ void __launch_bounds__(256) grad_sumsq_kernel(const float* g, int64_t n,
                                                         float* partials) {
  float s = 0.f;
  const int64_t n4 = (reinterpret_cast<uintptr_t>(g) & 15) == 0 ? n / 4 : 0;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 q = g4[i];
    s = fmaf(q.x, q.x, s);
    s = fmaf(q.y, q.y, s);
    s = fmaf(q.z, q.z, s);
    s = fmaf(q.w, q.w, s);
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    s = fmaf(g[i], g[i], s);
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    partials[blockIdx.x] = t;
  }
}

// One block: norm = sqrt(sum of the partials in block order), clip
// coefficient = min(1, max_norm / (norm + 1e-6)) as torch's clip_grad_norm_.
__global__ void __launch_bounds__(32) grad_clip_coef_kernel(const float* partials, int nparts,
                                                            float max_norm, float* out) {
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += 32) s += partials[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (threadIdx.x == 0) {
    const float norm = sqrtf(s);
    out[0] = norm;
    out[1] = fminf(__fdiv_rn(max_norm, __fadd_rn(norm, 1e-6f)), 1.f);
  }
}

// Backward of the Rosa output path into the payload (training hard path,
// rosa.py:164-165 under the Int8Linear STE of out_proj, linear.py:88-94): with
// gx = dL/d(dequantised out_proj input) (M, S) fp32, o = payload * sign (the
// out_proj input) and its GS128 codes, the STE input gradient is
//   do = gx + [|o| == amax_g] sign(o) fp16(sum_g gx * codes) / 127 / n_tied
// (the scale gradient of quant.py:47-49, only inside the clamp range), and
//   d payload[s] = sum_t do[t, s] * sign[t, s].
// One warp per 128-stream group (the last one zero-padded when S % 128 != 0,
// as quantize_last_dim pads), a thread owns 4 streams; CTA rows
// [blockIdx.x * rpc, +rpc); per-CTA column sums into partials (gridDim, S).
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__global__ void __launch_bounds__(512) rosa_payload_bwd_kernel(
    const T* __restrict__ o, const int8_t* __restrict__ codes, const float* __restrict__ gx,
    const T* __restrict__ sign, int64_t m, int S, int64_t rpc, float* __restrict__ partials) {
  const int tid = threadIdx.x;
  const int col = tid * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t r0 = (int64_t)blockIdx.x * rpc;
  const int64_t r1 = min(m, r0 + rpc);
  const bool live = col < S;  // S % 4 == 0: a thread's 4 streams are all real or all padding
  for (int64_t row = r0; row < r1; ++row) {
    const int64_t off = row * S + col;
    float ov[4] = {0.f, 0.f, 0.f, 0.f}, sv[4] = {0.f, 0.f, 0.f, 0.f};
    float gv[4] = {0.f, 0.f, 0.f, 0.f}, cv[4] = {0.f, 0.f, 0.f, 0.f};
    if (live) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ov[i] = to_f32(o[off + i]);
        sv[i] = to_f32(sign[off + i]);
      }
      const float4 g4 = *reinterpret_cast<const float4*>(gx + off);
      gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
      const char4 c4 = *reinterpret_cast<const char4*>(codes + off);
      cv[0] = c4.x; cv[1] = c4.y; cv[2] = c4.z; cv[3] = c4.w;
    }
    float am = 0.f, dot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      am = fmaxf(am, fabsf(ov[i]));
      dot += gv[i] * cv[i];
    }
    am = warp_max(am);
    dot = warp_sum(dot);
    float nt = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) nt += fabsf(ov[i]) == am ? 1.f : 0.f;
    nt = warp_sum(nt);
    const float g16 = __half2float(__float2half_rn(dot));
    const float s32 = am / 127.f;
    const bool inside = s32 >= 5.9604644775390625e-08f && s32 <= 65504.f;
    const float share = inside ? g16 / 127.f / nt : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float sg = ov[i] > 0.f ? 1.f : (ov[i] < 0.f ? -1.f : 0.f);
      const float d = gv[i] + (fabsf(ov[i]) == am ? sg * share : 0.f);
      acc[i] += d * sv[i];
    }
  }
  if (live) {
    float* pp = partials + (int64_t)blockIdx.x * S + col;
#pragma unroll
    for (int i = 0; i < 4; ++i) pp[i] = acc[i];
  }
}

// ---------------------------------------------------------------- counterfactual credits
//
// HardRosaGPU's backward (ksdraft/kernels/rosa_credit_gpu.py:25-48): for every
// q, k and v bit of a stream, flip it, re-match the whole window and sum
// (sign' - sign) * grad over the positions, grad = dL/d sign.  The reference
// builds all 3T perturbed streams and re-matches each in full (T <= 63); here
// only what a flip can change is recomputed, exactly:
//   v[p]  the sign of the positions whose match ends at p - 1 (closed form);
//   q[p]  the queries t in [p, p + 61] whose window has bit p at depth
//         l = t - p <= their match length (a shallower bit cannot change a
//         capped match): one full re-match each;
//   k[p]  the keys j in [p, p + 63] (their windows hold k[p] at depth j - p).
//         For a query t > p whose best key is not one of them, or is one whose
//         capped length does not drop, the new answer is the better of the old
//         one and the 64 changed keys; otherwise one full re-match with k[p]
//         flipped.  A query whose best key is later than every changed key and
//         already at the cap cannot change.
// One CTA per stream: 8 warps share the stream's words, gradients and base
// matches in shared memory; warp w takes the flips p = w, w + 8, ...
struct CreditArgs {
  const uint64_t* qw;
  const uint64_t* kw;
  const uint64_t* vw;
  const float* grad;   // (rows, T) dL/d sign
  float* cq;           // (rows, T) credits of the q, k, v bits
  float* ck;
  float* cv;
  int64_t rows, t_len;
  int max_len;
};

constexpr int CR_WARPS = 8;

// longest capped match of query window wq at t against keys j <= t - 1, the
// latest among the longest (bit-parallel per k word, as rosa_match_bits_kernel);
// fp >= 0: the k bit at position fp reads flipped
__device__ __forceinline__ int credit_match(const uint64_t* sk, int64_t t, uint64_t wq, int cap,
                                            int64_t fp, int64_t& bestj) {
  int best = 0;
  bestj = -1;
  if (cap <= 0) return 0;
  const int64_t fw = fp >= 0 ? (fp >> 6) : -1;
  const uint64_t fm = fp >= 0 ? (1ull << (fp & 63)) : 0ull;
  auto kword = [&](int64_t w) -> uint64_t { return sk[w] ^ (w == fw ? fm : 0ull); };
  const int64_t wl = (t - 1) >> 6;
  uint64_t M = ~0ull >> (63 - (int)((t - 1) & 63));
  for (int64_t w = wl; w >= 1; --w) {
    uint64_t mo;
    const int len = bits_word_match(kword(w), kword(w - 1), M, wq, cap, false, mo);
    if (len > best) {
      best = len;
      bestj = (w << 6) + 63 - __clzll((long long)mo);
      if (best == cap) return best;
    }
    M = ~0ull;
  }
  uint64_t mo;
  const int len = bits_word_match(kword(0), 0ull, wl == 0 ? M : ~0ull, wq, cap, true, mo);
  if (len > best) {
    best = len;
    bestj = 63 - __clzll((long long)mo);
  }
  return best;
}

__device__ __forceinline__ float credit_sign(const uint64_t* sv, int64_t j) {
  if (j < 0) return -1.f;
  const int64_t s = j + 1;
  return ((sv[s >> 6] >> (s & 63)) & 1ull) ? 1.f : -1.f;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(CR_WARPS * 32) rosa_credits_kernel(CreditArgs a) {
  extern __shared__ __align__(16) uint8_t crs[];
  const int64_t row = blockIdx.x;
  const int T = (int)a.t_len;
  const int nw = (T + 63) / 64;
  const int ml = a.max_len;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* sq = reinterpret_cast<uint64_t*>(crs);
  uint64_t* sk = sq + nw;
  uint64_t* sv = sk + nw;
  uint64_t* cw_all = sv + nw;                                   // [CR_WARPS][64] changed windows
  float* g = reinterpret_cast<float*>(cw_all + CR_WARPS * 64);  // [T]
  int16_t* bj = reinterpret_cast<int16_t*>(g + T);              // [T] base endpoints
  int8_t* bl = reinterpret_cast<int8_t*>(bj + T);               // [T] base lengths
  for (int i = threadIdx.x; i < nw; i += blockDim.x) {
    sq[i] = a.qw[row * nw + i];
    sk[i] = a.kw[row * nw + i];
    sv[i] = a.vw[row * nw + i];
  }
  for (int i = threadIdx.x; i < T; i += blockDim.x) g[i] = a.grad[row * T + i];
  __syncthreads();
  // base matches
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    int64_t j;
    const int len = credit_match(sk, t, window_sm(sq, t), min(ml, t), -1, j);
    bl[t] = (int8_t)len;
    bj[t] = (int16_t)j;
  }
  __syncthreads();
  // v[p]: positions whose match ends at p - 1 read their sign from v[p]
  for (int p = threadIdx.x; p < T; p += blockDim.x) {
    float c = 0.f;
    const float s = ((sv[p >> 6] >> (p & 63)) & 1ull) ? 1.f : -1.f;
    for (int t = 0; t < T; ++t)
      if (bj[t] >= 0 && bj[t] + 1 == p) c += (-2.f * s) * g[t];
    a.cv[row * T + p] = c;
  }
  // q[p]: queries t = p .. p + 61 whose window holds bit p at depth <= their length
  for (int p = warp; p < T; p += CR_WARPS) {
    float c = 0.f;
#pragma unroll
    for (int r = 0; r < 64; r += 32) {
      const int t = p + r + lane;
      const int l = r + lane;
      if (t < T) {
        const int cap = min(ml, t);
        if (l < cap && l <= bl[t]) {
          const uint64_t wq = window_sm(sq, t) ^ (1ull << (63 - l));
          int64_t nj;
          credit_match(sk, t, wq, cap, -1, nj);
          c += (credit_sign(sv, nj) - credit_sign(sv, bj[t])) * g[t];
        }
      }
    }
    c = warp_sum_f(c);
    if (lane == 0) a.cq[row * T + p] = c;
  }
  // k[p]: keys p .. p + 63 change
  uint64_t* cw = cw_all + warp * 64;
  for (int p = warp; p < T; p += CR_WARPS) {
#pragma unroll
    for (int r = 0; r < 64; r += 32) {
      const int j = p + r + lane;
      cw[r + lane] = j < T ? (window_sm(sk, j) ^ (1ull << (63 - (r + lane)))) : 0ull;
    }
    __syncwarp();
    float c = 0.f;
    for (int t = p + 1 + lane; t < T; t += 32) {
      const int cap = min(ml, t);
      const int best = bl[t];
      const int64_t bestj = bj[t];
      if (best == cap && bestj > p + 63) continue;   // a later key already at the cap
      const uint64_t wq = window_sm(sq, t);
      int nb = best;
      int64_t nbj = bestj;
      bool full = false;
      if (bestj >= p && bestj <= p + 63) {
        const uint64_t x = wq ^ cw[bestj - p];
        const int raw = x ? __clzll((long long)x) : 64;
        full = min(raw, min(cap, (int)bestj + 1)) < best;
      }
      if (full) {
        nb = credit_match(sk, t, wq, cap, p, nbj);
      } else {
        const int hi = min(63, t - 1 - p);
        for (int i = 0; i <= hi; ++i) {
          const int64_t j = p + i;
          const uint64_t x = wq ^ cw[i];
          int len = x ? __clzll((long long)x) : 64;
          len = min(len, min(cap, (int)j + 1));
          if (len > nb || (len == nb && len > 0 && j > nbj)) {
            nb = len;
            nbj = j;
          }
        }
      }
      c += (credit_sign(sv, nbj) - credit_sign(sv, bestj)) * g[t];
    }
    c = warp_sum_f(c);
    if (lane == 0) a.ck[row * T + p] = c;
    __syncwarp();   // cw is rewritten for the next p
  }
}

}  // namespace ksd8

using namespace ksd8;

int ksd8_rosa_payload_bwd_launch(const void* o, const int8_t* codes, const float* gx,
                                 const void* sign, int dtype, int64_t m, int64_t streams,
                                 float* partials, int64_t n_parts, cudaStream_t stream) {
  if (m == 0) {
    return cudaMemsetAsync(partials, 0, sizeof(float) * n_parts * streams, stream) == cudaSuccess
               ? KSD8_OK : KSD8_ERR_LAUNCH;
  }
  const int64_t rpc = (m + n_parts - 1) / n_parts;
  const unsigned threads = (unsigned)((streams + 127) / 128 * 32);  // whole warps per group
  switch (dtype) {
    case KSD8_F32:
      rosa_payload_bwd_kernel<float><<<(unsigned)n_parts, threads, 0, stream>>>(
          (const float*)o, codes, gx, (const float*)sign, m, (int)streams, rpc, partials);
      break;
    case KSD8_BF16:
      rosa_payload_bwd_kernel<__nv_bfloat16><<<(unsigned)n_parts, threads, 0, stream>>>(
          (const __nv_bfloat16*)o, codes, gx, (const __nv_bfloat16*)sign, m, (int)streams, rpc,
          partials);
      break;
    case KSD8_F16:
      rosa_payload_bwd_kernel<__half><<<(unsigned)n_parts, threads, 0, stream>>>(
          (const __half*)o, codes, gx, (const __half*)sign, m, (int)streams, rpc, partials);
      break;
    default:
      return KSD8_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}

int ksd8_adamw_multi_launch(int count, float* const* params, const void* const* grads, int gdt,
                            float* const* m, float* const* v, const int64_t* numels, float lr,
                            float b1, float b2, float eps, float wd, int step,
                            const float* gscale, cudaStream_t stream) {
  AdamwMulti t;
  int64_t total = 0;
  t.count = count;
  for (int k = 0; k < count; ++k) {
    t.p[k] = params[k];
    t.g[k] = grads[k];
    t.m[k] = m[k];
    t.v[k] = v[k];
    t.n[k] = numels[k];
    total += numels[k];
  }
  if (total == 0) return KSD8_OK;
  const float bc1 = 1.f - powf(b1, (float)step);
  const float bc2 = 1.f - powf(b2, (float)step);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  adamw_multi_kernel<<<(unsigned)blocks, 256, 0, stream>>>(t, gdt, lr, b1, b2, eps, wd, bc1,
                                                            sqrtf(bc2), gscale);
  return KSD8_OK;
}

int ksd8_grad_clip_launch(const float* grad, int64_t n, float max_norm, float* scratch,
                          float* out, cudaStream_t stream) {
  int64_t blocks = (n + 1023) / 1024;
  if (blocks < 1) blocks = 1;
  if (blocks > GN_BLOCKS) blocks = GN_BLOCKS;
  grad_sumsq_kernel<<<(unsigned)blocks, 256, 0, stream>>>(grad, n, scratch);
  grad_clip_coef_kernel<<<1, 32, 0, stream>>>(scratch, (int)blocks, max_norm, out);
  return KSD8_OK;
}

int ksd8_rosa_pack_bits_launch(const void* x, int x_dtype, int64_t batch, int64_t t_len,
                               int64_t streams, int64_t sb, int64_t st, int64_t ss,
                               uint64_t* words, cudaStream_t stream) {
  const int64_t total = batch * streams * ((t_len + 63) / 64);
  if (total == 0) return KSD8_OK;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  switch (x_dtype) {
    case KSD8_F32:
      rosa_pack_bits_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(
          reinterpret_cast<const float*>(x), batch, t_len, streams, sb, st, ss, words);
      break;
    case KSD8_F16:
      rosa_pack_bits_kernel<__half><<<(unsigned)blocks, 256, 0, stream>>>(
          reinterpret_cast<const __half*>(x), batch, t_len, streams, sb, st, ss, words);
      break;
    case KSD8_BF16:
      rosa_pack_bits_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
          reinterpret_cast<const __nv_bfloat16*>(x), batch, t_len, streams, sb, st, ss, words);
      break;
    case KSD8_I8:
      rosa_pack_bits_kernel<int8_t><<<(unsigned)blocks, 256, 0, stream>>>(
          reinterpret_cast<const int8_t*>(x), batch, t_len, streams, sb, st, ss, words);
      break;
    default:
      return KSD8_ERR_DTYPE;
  }
  return KSD8_OK;
}

// Matcher selection (process-wide): 0 = chunked prefix tables with the
// degenerate streams redone by the sorted-key kernel (default), 1 = one
// position per step prefix tables, 2 = window scan, 3 = sorted keys (streams
// up to 4096 + max_len - 1 positions, else as 0), 4 = bit-parallel for every
// stream.  Streams of 8192 or more positions take the bit-parallel kernel
// (the window scan under 2).  algo < 0 only reads.
// Config-4 layer (16 x 2048 positions x 512 streams): fair bits 2.28 ms
// (0) / 6.59 (3) / 3.60 (4); bits in runs of ~10 (deep layers) 7.30 / 6.42 /
// 7.59 ms; the bit-parallel kernel as the redo pass of 0 gave 8.47 ms there.
// 512 streams of 8192 / 16384 positions, window scan vs bit-parallel: fair
// bits 21.7 / 13.0 and 115.9 / 51.1 ms, runs 21.5 / 27.1 and 115.6 / 107.8 ms.
int ksd8_rosa_algorithm(int algo) {
  static int g_algo = 0;
  if (algo >= 0 && algo <= 4) g_algo = algo;
  return g_algo;
}

// The bit-parallel matcher over the given streams (all, or the redo list).
static int launch_bits(const MatchArgs& a, int64_t n, cudaStream_t stream) {
  const int nw = (int)((a.t_len + 63) / 64);
  const size_t per_warp = (size_t)3 * nw * 8;
  int nwarps = 8;
  while (nwarps > 1 && (size_t)nwarps * per_warp > 227 * 1024) nwarps >>= 1;
  const size_t smem = (size_t)nwarps * per_warp;
  if (smem > 227 * 1024) return KSD8_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    static unsigned attr = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 32) return KSD8_ERR_UNSUPPORTED;
    if (!(attr & (1u << dev))) {
      if (cudaFuncSetAttribute(rosa_match_bits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               227 * 1024) != cudaSuccess)
        return KSD8_ERR_LAUNCH;
      attr |= 1u << dev;
    }
  }
  rosa_match_bits_kernel<<<(unsigned)((n + nwarps - 1) / nwarps), nwarps * 32, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}


// The prefix-table matchers (chunked, or one position per step for algo 1).
static int launch_chunk(const MatchArgs& a, int64_t t_len, int dev, int algo,
                        cudaStream_t stream) {
  static unsigned prefix_attr = 0;
  // bytes per warp: tables + links (16-byte aligned), then 3 x ceil(T/64) words
  // (a multiple of 16 bytes, so that every warp's region keeps the 16-byte
  // alignment of its vector stores)
  const int stride = (int)(((((size_t)RP_TBL + t_len) * 2 + 15) / 16 * 16 +
                            3 * 8 * (size_t)((t_len + 63) / 64) + 15) / 16 * 16);
  int nwarps = (int)((227 * 1024) / (size_t)stride);
  const int cap_warps = algo == 1 ? RP_WARPS : RC_WARPS;
  if (nwarps > cap_warps) nwarps = cap_warps;
  const size_t psmem = (size_t)nwarps * stride;
  if (!(prefix_attr & (1u << dev))) {
    if (cudaFuncSetAttribute(rosa_match_prefix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(rosa_match_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    prefix_attr |= (1u << dev);
  }
  const int64_t n = a.batch * a.streams;
  const unsigned grid = (unsigned)((n + nwarps - 1) / nwarps);
  if (algo == 1)
    rosa_match_prefix_kernel<<<grid, nwarps * 32, psmem, stream>>>(a, stride);
  else
    rosa_match_chunk_kernel<<<grid, nwarps * 32, psmem, stream>>>(a, stride);
  return KSD8_OK;
}

#ifndef KSD8_ROSA_REDO_BUDGET
#define KSD8_ROSA_REDO_BUDGET 8
#endif

// Chain steps per position (average, after the first 96 positions) that the
// chunked matcher spends on a stream before handing it to the sorted-key one;
// KSD8_ROSA_REDO_BUDGET in the environment overrides the compiled default.
// Config-4 step, Rosa forward of the 24 layers: 149.8 / 151.2 / 140.2 / 156.4 /
// 184.6 ms at budgets 2 / 4 / 8 / 16 / 32.
static int redo_budget() {
  static const int b = [] {
    const char* e = std::getenv("KSD8_ROSA_REDO_BUDGET");
    const int v = e ? std::atoi(e) : 0;
    return v > 0 ? v : KSD8_ROSA_REDO_BUDGET;
  }();
  return b;
}

int ksd8_rosa_match_launch(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw,
                           int64_t batch, int64_t streams, int64_t t_len, int max_len,
                           const float* payload, void* out, int out_dtype, int64_t ob, int64_t ot,
                           int64_t os, int32_t* match_len, int32_t* match_end,
                           cudaStream_t stream, int32_t* redo) {
  if (batch * streams == 0 || t_len == 0) return KSD8_OK;
  const size_t smem = (size_t)t_len * 8;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && !(attr_dev_mask & (1 << dev))) {
    if (cudaFuncSetAttribute(rosa_match_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024) != cudaSuccess)
      return KSD8_ERR_LAUNCH;
    attr_dev_mask |= (1 << dev);
  }
  MatchArgs a;
  a.qw = qw; a.kw = kw; a.vw = vw; a.batch = batch; a.streams = streams; a.t_len = t_len;
  a.max_len = max_len; a.payload = payload; a.out = out; a.out_dtype = out_dtype;
  a.ob = ob; a.ot = ot; a.os = os; a.match_len = match_len; a.match_end = match_end;
  a.redo = nullptr; a.redo_budget = 0; a.redo_pass = 0;
  const int algo = ksd8_rosa_algorithm(-1);
  // the sorted-key matcher's per-warp shared memory (keys, tree, ranks, bitmap, words)
  const int r0 = max_len > 0 ? max_len - 1 : 0;
  const int64_t nk = t_len - 1 - r0 > 0 ? t_len - 1 - r0 : 0;
  int np = 64;
  while (np < nk) np <<= 1;
  const bool sorted_ok = np <= RS_MAXNP;
  if (algo == 0 && redo && sorted_ok && t_len < RP_TMAX) {
    // adaptive: chunked prefix tables, degenerate streams redone by the sorted kernel
    if (cudaMemsetAsync(redo, 0, sizeof(int32_t), stream) != cudaSuccess) return KSD8_ERR_LAUNCH;
    a.redo = redo;
    a.redo_budget = redo_budget();
  }
  if (algo == 4) return launch_bits(a, batch * streams, stream);
  if (algo == 3 || a.redo) {
    if (sorted_ok) {
      const size_t head = ((size_t)np * 12 + (size_t)t_len * 2 + 15) / 16 * 16;
      const int stride = (int)((head + np / 8 + 16 + 24 * (size_t)((t_len + 63) / 64) + 512 +
                                15) / 16 * 16);
      int nwarps = (int)((227 * 1024) / (size_t)stride);
      if (nwarps > RC_WARPS) nwarps = RC_WARPS;
      if (nwarps >= 1) {
        static unsigned sorted_attr = 0;
        if (!(sorted_attr & (1u << dev))) {
          if (cudaFuncSetAttribute(rosa_match_sorted_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
              cudaSuccess)
            return KSD8_ERR_LAUNCH;
          sorted_attr |= (1u << dev);
        }
        const int64_t n = batch * streams;
        if (!a.redo) {
          rosa_match_sorted_kernel<<<(unsigned)((n + nwarps - 1) / nwarps), nwarps * 32,
                                     (size_t)nwarps * stride, stream>>>(a, np, stride);
          return KSD8_OK;
        }
        // adaptive: the chunked kernel first (below), then the listed streams here
        const int rc = launch_chunk(a, t_len, dev, algo, stream);
        if (rc != KSD8_OK) return rc;
        MatchArgs r = a;
        r.redo_pass = 1;
        rosa_match_sorted_kernel<<<(unsigned)((n + nwarps - 1) / nwarps), nwarps * 32,
                                   (size_t)nwarps * stride, stream>>>(r, np, stride);
        return KSD8_OK;
      }
    }
    a.redo = nullptr;
  }
  if (t_len < RP_TMAX && algo != 2) return launch_chunk(a, t_len, dev, algo, stream);
  if (algo != 2) return launch_bits(a, batch * streams, stream);
  int threads = 512;
  if (t_len <= 256) threads = 256;
  rosa_match_kernel<<<(unsigned)(batch * streams), threads, smem, stream>>>(a);
  return KSD8_OK;
}

int ksd8_rosa_timemix_launch(const void* x, int x_dtype, int64_t batch, int64_t t_len, int64_t d,
                             const float* mq, const float* mk, const float* mv, int8_t* qc,
                             void* qs, int8_t* kc, void* ks, int8_t* vc, void* vs,
                             cudaStream_t stream) {
  TimemixArgs a;
  a.x = x; a.batch = batch; a.t_len = t_len; a.d = d;
  a.mix[0] = mq; a.mix[1] = mk; a.mix[2] = mv;
  a.codes[0] = qc; a.codes[1] = kc; a.codes[2] = vc;
  a.scales[0] = reinterpret_cast<__half*>(qs);
  a.scales[1] = reinterpret_cast<__half*>(ks);
  a.scales[2] = reinterpret_cast<__half*>(vs);
  const int64_t work = (batch * t_len + TM_TOKENS - 1) / TM_TOKENS * ((d + 127) / 128);
  if (work == 0 || d == 0) return KSD8_OK;
  int64_t blocks = (work + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  switch (x_dtype) {
    case KSD8_F32: rosa_timemix_quant_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    case KSD8_BF16:
      rosa_timemix_quant_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(a);
      break;
    case KSD8_F16: rosa_timemix_quant_kernel<__half><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    default: return KSD8_ERR_DTYPE;
  }
  return KSD8_OK;
}

int ksd8_adamw_launch(float* p, const void* g, int gdt, float* m, float* v, int64_t n, float lr,
                      float b1, float b2, float eps, float wd, int step, cudaStream_t stream,
                      const float* gscale) {
  if (n == 0) return KSD8_OK;
  const float bc1 = 1.f - powf(b1, (float)step);
  const float bc2 = 1.f - powf(b2, (float)step);
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  adamw_kernel<<<(unsigned)blocks, 256, 0, stream>>>(p, g, gdt, m, v, n, lr, b1, b2, eps, wd, bc1,
                                                      sqrtf(bc2), gscale);
  return KSD8_OK;
}

// shared memory of rosa_credits_kernel for a stream of t_len positions
static size_t credits_smem(int64_t t_len) {
  const int64_t nw = (t_len + 63) / 64;
  return (size_t)(3 * nw + CR_WARPS * 64) * 8 + (size_t)t_len * (4 + 2 + 1) + 16;
}

int ksd8_rosa_credits_launch(const uint64_t* qw, const uint64_t* kw, const uint64_t* vw,
                             int64_t rows, int64_t t_len, int max_len, const float* grad,
                             float* cq, float* ck, float* cv, cudaStream_t stream) {
  if (rows == 0 || t_len == 0) return KSD8_OK;
  const size_t smem = credits_smem(t_len);
  if (smem > 227 * 1024) return KSD8_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    static unsigned attr = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 32) return KSD8_ERR_UNSUPPORTED;
    if (!(attr & (1u << dev))) {
      if (cudaFuncSetAttribute(rosa_credits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               227 * 1024) != cudaSuccess)
        return KSD8_ERR_LAUNCH;
      attr |= 1u << dev;
    }
  }
  CreditArgs a;
  a.qw = qw; a.kw = kw; a.vw = vw; a.grad = grad; a.cq = cq; a.ck = ck; a.cv = cv;
  a.rows = rows; a.t_len = t_len; a.max_len = max_len;
  rosa_credits_kernel<<<(unsigned)rows, CR_WARPS * 32, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? KSD8_OK : KSD8_ERR_LAUNCH;
}
