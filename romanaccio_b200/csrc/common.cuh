// Device-side helpers shared by the W8A8 kernels (sm_100a).
//
// Numerics restated here:
//   round_clamp      round_clamp_f32, src/LFM3/lfm3_v2.cpp:248-257 (clamp, then round-half-even)
//   requant_quantm   SDP CvtPrecision_QuantM: clip(RNE(acc * QuantM / 2^trunc), +-Qmax)
//                    (src/LFM3/attribute_int8_error.py:104-122, FINDINGS.md:2447), done in exact
//                    int64 arithmetic; the reference's float64 product acc*(QuantM/2^trunc) is
//                    exact because |acc * QuantM| < 2^46, so both give the same integer.
//   topk_key         total order (value desc, vocab id asc) used for argmax / top-k
//                    (sampler.cpp:93-103 keeps the lowest id on ties).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace w8a8 {

// Upper bound for any spin wait inside a kernel: 2 seconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

// The "memory" clobber keeps the read in program order with barriers and memory operations.
__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t)::"memory");
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------
// mbarrier + bulk copy (TMA 1-D, no tensor map, one CTA per copy)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in *err) when the
// phase did not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int *err,
                                                  int code) {
  if (mbar_try_wait(bar, parity)) return true;
  // %globaltimer is slow to read: poll the barrier, and look at the clock every 512 polls.
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 511u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Cross-device flags (counters that only grow; compared modulo 2^32)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys(unsigned *p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's earlier generic-proxy accesses (an acquire included) before its later
// bulk copies, which read global memory through the async proxy.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until *flag reaches `target`.  Returns false (and records `code` in *err) after
// limit_ns of %globaltimer.
__device__ __forceinline__ bool wait_flag_reached(const unsigned *flag, unsigned target,
                                                  unsigned long long limit_ns, int *err, int code) {
  if (static_cast<int>(ld_acquire_sys(flag) - target) >= 0) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (static_cast<int>(ld_acquire_sys(flag) - target) >= 0) return true;
    if ((i & 255u) == 0 && global_timer_ns() - t0 > limit_ns) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

// Global -> shared bulk copy completing on an mbarrier (bytes multiple of 16, both addresses
// 16-byte aligned).  Streamed operands use an evict-first L2 policy.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------------------
// Programmatic dependent launch
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// Numerics
// ---------------------------------------------------------------------------------------
// std::min(std::max(x, -lim), lim) followed by round-half-even.  The comparisons are written
// as std::max / std::min evaluate them, so a NaN input stays NaN through the clamp and
// converts to 0 (as the x86 build of the reference yields for int8).
__device__ __forceinline__ int32_t round_clamp(float x, float lim) {
  float c = (x < -lim) ? -lim : x;
  c = (lim < c) ? lim : c;
  return __float2int_rn(c);
}

// Round-half-even of p / 2^trunc with one add and one arithmetic shift: with p = f * 2^t + r
// (0 <= r < 2^t), adding 2^(t-1) - 1 + (f & 1) carries into f exactly when r > 2^(t-1), or when
// r == 2^(t-1) and f is odd.
__device__ __forceinline__ int32_t requant_quantm(int32_t acc, int32_t qm, int32_t trunc,
                                                  int32_t qmax) {
  const long long p = static_cast<long long>(acc) * static_cast<long long>(qm);
  long long q = p;
  if (trunc > 0) {
    const long long odd = (p >> trunc) & 1LL;
    q = (p + ((1LL << (trunc - 1)) - 1) + odd) >> trunc;
  }
  q = q < -qmax ? -qmax : (q > qmax ? qmax : q);
  return static_cast<int32_t>(q);
}

// requant_quantm for 15 <= trunc <= 31, where the quotient fits 32 bits (|acc * QuantM| < 2^46):
// the low words of the shifts come from 32-bit funnel shifts of the 64-bit product (the low 32
// bits of a logical and an arithmetic shift agree).  bias = 2^(trunc-1) - 1.
__device__ __forceinline__ int32_t requant_quantm_t15(int32_t acc, int32_t qm, int32_t trunc,
                                                      long long bias, int32_t qmax) {
  const long long p = static_cast<long long>(acc) * static_cast<long long>(qm);
  const uint32_t odd =
      __funnelshift_r(static_cast<uint32_t>(p), static_cast<uint32_t>(p >> 32), trunc) & 1u;
  const long long r = p + bias + odd;
  int32_t q = static_cast<int32_t>(
      __funnelshift_r(static_cast<uint32_t>(r), static_cast<uint32_t>(r >> 32), trunc));
  q = q < -qmax ? -qmax : (q > qmax ? qmax : q);
  return q;
}

// The same requant in float64, the reference's own formulation (round(acc * (QuantM / 2^trunc))):
// scale = QuantM * 2^-trunc is exact, and so is acc * scale because |acc * QuantM| < 2^46 fits
// the 53-bit significand; clamping to the integer bound before the round-half-even conversion
// gives the same integer as clipping after it.  Five instructions instead of the int64 chain.
__device__ __forceinline__ double quantm_scale(int32_t qm, int32_t trunc) {
  // 2^-trunc built from its exponent bits (trunc in [0, 62])
  return static_cast<double>(qm) * __longlong_as_double(static_cast<long long>(1023 - trunc) << 52);
}

__device__ __forceinline__ int32_t requant_f64(int32_t acc, double scale, double qmax) {
  double x = static_cast<double>(acc) * scale;
  x = x < -qmax ? -qmax : x;
  x = x > qmax ? qmax : x;
  return __double2int_rn(x);
}

__device__ __forceinline__ uint64_t topk_key(float v, uint32_t id) {
  uint32_t u = __float_as_uint(v);
  if ((u << 1) == 0u) u = 0u;  // -0.0 and +0.0 compare equal in the reference
  const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<uint64_t>(o) << 32) | static_cast<uint64_t>(0xFFFFFFFFu - id);
}

__device__ __forceinline__ float topk_key_value(uint64_t key) {
  const uint32_t o = static_cast<uint32_t>(key >> 32);
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(u);
}

__device__ __forceinline__ int32_t topk_key_id(uint64_t key) {
  return static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key));
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Max over non-NaN values in the style of `if (a > amax) amax = a`.
__device__ __forceinline__ float warp_amax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = (w > v) ? w : v;
  }
  return v;
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = (w > v) ? w : v;
  }
  return v;
}

}  // namespace w8a8
