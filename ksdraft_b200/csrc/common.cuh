// Shared device helpers for the ksd8 sm_100a kernels.
//
// Everything here is plain CUDA / inline PTX for Blackwell (sm_100a):
// mbarrier waits with a wall-clock bound, TMA (cp.async.bulk.tensor) loads
// without multicast, tcgen05 (TMEM alloc / MMA / ld / commit) wrappers.
//
// Every spin-wait is bounded: after KSD8_WAIT_NS nanoseconds of global timer
// time a wait gives up, records KSD8_ERR_DEVICE_TIMEOUT in the status word the
// host passed in and reports failure to its caller, which then drains and
// exits instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/ksd8.h"

// Host: grid of a persistent kernel, leaving ksd8_get_sm_reserve() SMs to
// concurrent collectives (capi.cu holds the setting).
static inline int ksd8_persistent_ctas(int sm_count) {
  const int n = sm_count - ksd8_get_sm_reserve();
  return n < 1 ? 1 : n;
}

#ifndef KSD8_SUSPEND_NS
#define KSD8_SUSPEND_NS 20000u  // suspend-time hint of one try_wait (woken on completion)
#endif
#ifndef KSD8_WAIT_NS
#define KSD8_WAIT_NS 2000000000ull  // 2 s of global-timer time per wait
#endif
#ifndef KSD8_WAIT_BACKOFF_NS
#define KSD8_WAIT_BACKOFF_NS 0      // optional __nanosleep between polls of a bounded wait
#endif

namespace ksd8 {

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a warp whose phase is not complete is
// parked (up to `ns` nanoseconds, woken when the phase completes) instead of
// re-issuing the test, so waiting warps leave the issue slots of their SM
// sub-partition to the warps that compute.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait. Returns false (and records a timeout) when the phase did not
// complete within KSD8_WAIT_NS, or when another warp of the CTA already gave
// up (abort flag in shared memory), so that every role drains promptly.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, KSD8_SUSPEND_NS)) return true;
    if (KSD8_WAIT_BACKOFF_NS) __nanosleep(KSD8_WAIT_BACKOFF_NS);
    if ((++n & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > KSD8_WAIT_NS) {
        *abort_flag = 1;
        record_error(status, KSD8_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D tiled TMA load global -> shared (this CTA), completion counted on `bar`.
// No multicast: every CTA fetches its own tiles.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy global -> shared (this CTA), completion counted on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_load_g2s(void* smem_dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes),
      "r"(smem_u32(bar))
      : "memory");
}

// 2D tiled TMA store shared (this CTA) -> global, tracked by the issuing
// thread's bulk async-group.  Elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src,
                                             int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// The issuing thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// ... and have completed (global writes performed).
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic-proxy accesses of shared memory before later
// async-proxy (TMA) accesses of the same bytes (a buffer refilled by TMA
// after threads read or wrote it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Host: SM count of the current device (cached per device).
static inline int current_sm_count() {
  static int n[32] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 32) return 148;
  if (!n[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    n[dev] = v;
  }
  return n[dev];
}

// Host: cuTensorMapEncodeTiled through the runtime's driver entry point
// (no link-time dependency on libcuda).
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static inline PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}


// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every previously issued tcgen05 op of this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives lane
// (taddr.lane + t), columns taddr.col .. taddr.col+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

template <int W>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[W]) {
  if constexpr (W == 32) tmem_ld_32x32b_x32(taddr, r);
  else tmem_ld_32x32b_x16(taddr, r);
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms):
// start address, stride between 8-row groups (SBO = 1024 B), descriptor
// version 1 (sm100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_k128_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);          // start address
  d |= (uint64_t)(1u) << 16;                         // leading byte offset (unused when swizzled)
  d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;     // stride byte offset
  d |= (uint64_t)1u << 46;                           // version
  d |= (uint64_t)2u << 61;                           // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::i8: D = s32, A = B = signed int8, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// ---------------------------------------------------------------- misc math

// Exact int32 -> fp32 for |v| < 2^22 without the conversion pipe: the integer
// is added to the bit pattern of 1.5 * 2^23 and the offset subtracted in fp32.
__device__ __forceinline__ float i2f_exact22(int32_t v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// GS128 scale: fp32 amax/127 (IEEE division), clamped to [2^-24, 65504], then
// rounded through fp16 so encode and decode use the same value.
__device__ __forceinline__ float gs_scale(float amax, __half* out_h) {
  float s = __fdiv_rn(amax, 127.0f);
  s = fminf(fmaxf(s, 5.9604644775390625e-08f), 65504.0f);
  __half h = __float2half_rn(s);
  if (out_h) *out_h = h;
  return __half2float(h);
}

// max that propagates NaN (a NaN distance sends the value to the exact path).
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Symmetric int8 code: round-half-even(x / scale), saturated to [-127, 127].
__device__ __forceinline__ int gs_code(float x, float scale) {
  float q = rintf(__fdiv_rn(x, scale));
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return (int)q;
}

// Same result as gs_code without a division on the common path.  y = x * rcp
// (rcp = RN(1/scale)) is within 2^-16 of RN(x/scale) for |x/scale| < 256, so
// rint(y) == rint(RN(x/scale)) unless y lies within 2^-14 of a half-integer;
// those (and out-of-range quotients) take the IEEE division.
// rcp may be the 1-ulp approximation of rcp_approx: |y - RN(x/scale)| then
// stays below 2^-14 for |y| < 200, and the margin used is 2^-13.  The integer
// is formed with the 1.5 * 2^23 shifter (round half to even, exact for
// |y| < 2^22) on the FMA/ALU pipes instead of the conversion unit.
// Out-of-line IEEE paths of the fast quantisers: rarely taken, kept out of the
// callers' hot loops so that those stay small in the instruction cache.
static __device__ __noinline__ int gs_code_slow(float x, float scale) { return gs_code(x, scale); }
static __device__ __noinline__ uint32_t gs_scale_slow_bits(float amax) {
  __half h;
  gs_scale(amax, &h);
  return __half_as_ushort(h);
}

__device__ __forceinline__ int gs_code_fast(float x, float scale, float rcp) {
  const float y = __fmul_rn(x, rcp);
  const float t = __fadd_rn(y, 12582912.f);
  const float r = __fsub_rn(t, 12582912.f);
  if (fabsf(y) < 200.f && fabsf(__fsub_rn(y, r)) < 0.4998779296875f) {  // 0.5 - 2^-13
    const int q = __float_as_int(t) - 0x4B400000;
    return min(max(q, -127), 127);
  }
  return gs_code_slow(x, scale);
}

// Four codes of one 128-wide group (common scale, rcp = RN(1/scale) within 1
// ulp), packed byte e = element e.  The scale is a normal fp16 number and not
// clamped above, so |y| <= 127.07: the 1.5 * 2^23 shifter's low byte is the
// code and no saturation applies; an element within 2^-13 of a rounding tie
// sends the four to the IEEE path.
static __device__ __noinline__ uint32_t gs_code4_exact(float x0, float x1, float x2, float x3,
                                                       float scale) {
  return ((uint32_t)gs_code(x0, scale) & 0xFFu) | (((uint32_t)gs_code(x1, scale) & 0xFFu) << 8) |
         (((uint32_t)gs_code(x2, scale) & 0xFFu) << 16) |
         (((uint32_t)gs_code(x3, scale) & 0xFFu) << 24);
}

__device__ __forceinline__ uint32_t gs_code4_normal(const float (&v)[4], float scale, float rcp) {
  const float2 rc = make_float2(rcp, rcp);
  const float2 mg = make_float2(12582912.f, 12582912.f), nmg = make_float2(-12582912.f, -12582912.f);
  const float2 y01 = __fmul2_rn(make_float2(v[0], v[1]), rc);
  const float2 y23 = __fmul2_rn(make_float2(v[2], v[3]), rc);
  const float2 t01 = __fadd2_rn(y01, mg), t23 = __fadd2_rn(y23, mg);
  const float2 d01 = __ffma2_rn(y01, make_float2(-1.f, -1.f), __fadd2_rn(t01, nmg));
  const float2 d23 = __ffma2_rn(y23, make_float2(-1.f, -1.f), __fadd2_rn(t23, nmg));
  const float dm =
      fmax_nan(fmax_nan(fabsf(d01.x), fabsf(d01.y)), fmax_nan(fabsf(d23.x), fabsf(d23.y)));
  if (!(dm < 0.4998779296875f)) return gs_code4_exact(v[0], v[1], v[2], v[3], scale);
  return __byte_perm(__byte_perm(__float_as_uint(t01.x), __float_as_uint(t01.y), 0x0040),
                     __byte_perm(__float_as_uint(t23.x), __float_as_uint(t23.y), 0x0040), 0x5410);
}

// Bounded wait of the staged quantisers: the mbarrier wait with a suspend hint
// by default; KSD8_Q_SPIN_WAIT polls without it (same bound, same abort).
__device__ __forceinline__ bool q_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                       int* status) {
#ifdef KSD8_Q_SPIN_WAIT
  uint64_t t0 = 0;
  for (uint32_t n = 0;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 63u) == 63u) {
      if (*abort_flag) return false;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      if (now - t0 > KSD8_WAIT_NS) {
        *abort_flag = 1;
        record_error(status, KSD8_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
#else
  return mbar_wait(bar, parity, abort_flag, status);
#endif
}

// True when gs_code4_normal applies to a group of amax `amax` and scale
// `scale`: the scale is a normal fp16 number not clamped above (or the group
// is all zeros).
__device__ __forceinline__ bool gs_scale_is_normal(float amax, float scale) {
  return !(amax > 0.f && (!(scale >= 6.103515625e-05f) || !(amax <= 8.0e6f)));
}

// 1/s to within 1 ulp (s a normal fp32; GS scales are >= 2^-24).
__device__ __forceinline__ float rcp_approx(float s) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
  return r;
}

// gs_scale without the division on the common path: y = amax * RN(1/127) is
// within 2.5 ulp of RN(amax/127); unless y sits within 4 ulp of an fp16
// rounding midpoint (or outside the normal fp16 range) fp16(y) is the exact
// answer, otherwise the IEEE path decides.
__device__ __forceinline__ float gs_scale_fast(float amax, __half* out_h) {
  const float y = __fmul_rn(amax, 0.007874015718698502f);
  const int low13 = (int)(__float_as_uint(y) & 0x1FFFu);
  if (y >= 6.103515625e-05f && y < 65504.f && abs(low13 - 0x1000) > 4) {
    const __half h = __float2half_rn(y);
    if (out_h) *out_h = h;
    return __half2float(h);
  }
  const __half h = __ushort_as_half((unsigned short)gs_scale_slow_bits(amax));
  if (out_h) *out_h = h;
  return __half2float(h);
}

// ---------------------------------------------------------------- Philox4x32-10
// Counter-based RNG of Salmon, Moraes, Dror and Shaw, "Parallel random
// numbers: as easy as 1, 2, 3" (SC'11): 10 rounds of the 4x32 Philox S-box
// with multipliers 0xD2511F53 / 0xCD9E8D57 and Weyl key increments
// 0x9E3779B9 / 0xBB67AE85.  Element `idx` of a stream keyed by `seed` is word
// (idx & 3) of the block at counter (idx >> 2, 0).
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0;
    const uint32_t n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
  }
}

// 24-bit uniform in [0, 1) of element idx: (word >> 8) * 2^-24.
__host__ __device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t idx) {
  uint32_t c[4] = {(uint32_t)(idx >> 2), (uint32_t)(idx >> 34), 0u, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(c[idx & 3] >> 8) * 5.9604644775390625e-08f;
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// Two CTAs of a cluster cooperate on one 256-row MMA: each stages half of the
// operands in its own shared memory, the even ("leader") CTA issues the MMA.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Arrive on the mbarrier at the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
      "r"(rank)
      : "memory");
}

// Shared::cluster address of this CTA's `p`, redirected to the leader (even) CTA of the pair.
__device__ __forceinline__ uint32_t leader_smem_addr(const void* p) {
  return smem_u32(p) & 0xFEFFFFFFu;
}

// 2D tiled TMA load into this CTA's shared memory whose completion is counted
// on the leader CTA's mbarrier (cta_group::2 form, no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T, issued by the leader.
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask` when
// the pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

}  // namespace ksd8
