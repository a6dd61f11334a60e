// Device helpers of the B200 sampler: Philox4x32-10, the correctly rounded
// binary32 exp, float ordering keys and warp collectives.
//
// Every binary32 operation that the reference performs (src/talker/sampling.rs)
// is written with an explicit round-to-nearest intrinsic (__fadd_rn,
// __fmul_rn, __fdiv_rn), so no multiply-add is ever contracted; the file is
// also compiled with -fmad=false.
#pragma once

#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace q3s {

constexpr unsigned FULL = 0xFFFFFFFFu;

// ---------------------------------------------------------------------------
// Philox4x32-10 (sampling.rs:12-17, 337-375): key = seed, counter =
// [ctr_lo, 0, subseq_lo, subseq_hi]; only word 0 feeds the uniform.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t philox_word0(uint64_t seed, uint64_t subseq, uint32_t ctr_lo) {
  uint32_t s0 = ctr_lo, s1 = 0u, s2 = (uint32_t)subseq, s3 = (uint32_t)(subseq >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t hi0 = __umulhi(0xD2511F53u, s0), lo0 = 0xD2511F53u * s0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, s2), lo1 = 0xCD9E8D57u * s2;
    const uint32_t n0 = hi1 ^ s1 ^ k0;
    const uint32_t n2 = hi0 ^ s3 ^ k1;
    s0 = n0;
    s1 = lo1;
    s2 = n2;
    s3 = lo0;
  }
  return s0;
}

// next_uniform (sampling.rs:373): ((w0 as f32) + 0.5) * 2^-32, in (0, 1].
__device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t subseq, uint32_t ctr_lo) {
  const uint32_t w = philox_word0(seed, subseq, ctr_lo);
  return __fmul_rn(__fadd_rn(__uint2float_rn(w), 0.5f), 2.3283064365386963e-10f);
}

// ---------------------------------------------------------------------------
// Correctly rounded binary32 exp.  Evaluated in binary64: k = rint(x/ln2),
// r = x - k*ln2 with a two-constant split (fused), exp(r) by its Taylor series
// to degree 13 in Horner form (|r| <= 0.347: truncation below 2^-57), scaled
// by 2^k and rounded once to binary32.  Checked bit for bit against long
// double expl over every binary32 in [-104, 0].
// ---------------------------------------------------------------------------
__device__ __forceinline__ float cr_expf(float xf) {
  if (xf != xf) return __fadd_rn(xf, xf);
  if (xf < -104.0f) return 0.0f;
  if (xf > 89.0f) return __int_as_float(0x7f800000);
  const double x = (double)xf;
  const double kd = rint(__dmul_rn(x, 0x1.71547652b82fep+0));
  double r = __fma_rn(-kd, 0x1.62e42fefa39efp-1, x);
  r = __fma_rn(-kd, 0x1.abc9e3b39803fp-56, r);
  double p = 0x1.6124613a86d09p-33;
  p = __fma_rn(p, r, 0x1.1eed8eff8d898p-29);
  p = __fma_rn(p, r, 0x1.ae64567f544e4p-26);
  p = __fma_rn(p, r, 0x1.27e4fb7789f5cp-22);
  p = __fma_rn(p, r, 0x1.71de3a556c734p-19);
  p = __fma_rn(p, r, 0x1.a01a01a01a01ap-16);
  p = __fma_rn(p, r, 0x1.a01a01a01a01ap-13);
  p = __fma_rn(p, r, 0x1.6c16c16c16c17p-10);
  p = __fma_rn(p, r, 0x1.1111111111111p-7);
  p = __fma_rn(p, r, 0x1.5555555555555p-5);
  p = __fma_rn(p, r, 0x1.5555555555555p-3);
  p = __fma_rn(p, r, 0.5);
  p = __fma_rn(p, r, 1.0);
  p = __fma_rn(p, r, 1.0);
  const long long k = (long long)kd;
  const double scale = __longlong_as_double((k + 1023LL) << 52);
  return __double2float_rn(__dmul_rn(p, scale));
}

// ---------------------------------------------------------------------------
// Ordering keys.
// ---------------------------------------------------------------------------
// Unsigned key whose integer order is the IEEE total order of binary32
// (f32::total_cmp; -0 < +0).
__device__ __forceinline__ uint32_t total_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return u ^ ((uint32_t)((int32_t)u >> 31) | 0x80000000u);
}
__device__ __forceinline__ float from_total_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

__device__ __forceinline__ bool is_finite(float v) { return fabsf(v) <= 3.40282347e38f; }

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// ---------------------------------------------------------------------------
// Warp collectives.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Maximum that ignores NaN (fmaxf semantics) and keeps +inf.
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
  return v;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(FULL, v, o);
    v = w > v ? w : v;
  }
  return v;
}

__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(FULL, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// Inclusive prefix sum over lanes.
__device__ __forceinline__ uint32_t warp_inclusive_scan(uint32_t v) {
  const unsigned lane = lane_id();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t w = __shfl_up_sync(FULL, v, o);
    if (lane >= (unsigned)o) v += w;
  }
  return v;
}

// ---------------------------------------------------------------------------
// Bulk copies (TMA, no multicast) completing on an mbarrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Makes generic-proxy shared-memory accesses (reads of a buffer, an
// mbarrier's initialisation) visible to the async proxy before a bulk copy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both ends 16-byte
// aligned) that signals `bar` on completion.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Test-and-sleep: the thread may be suspended up to `hint_ns` nanoseconds
// waiting for the phase, so a waiting warp issues almost nothing.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity,
                                              uint32_t hint_ns = 200000u) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` for at most ~`limit_ns` nanoseconds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (!mbar_try_wait(bar, parity)) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > limit_ns) return false;
  }
  return true;
}

// Element i of a row as binary32 (bf16 upcasts exactly).
template <int DTYPE>
__device__ __forceinline__ float load_elem(const void* base, int64_t i);

template <>
__device__ __forceinline__ float load_elem<0>(const void* base, int64_t i) {
  return __ldg(static_cast<const float*>(base) + i);
}

template <>
__device__ __forceinline__ float load_elem<1>(const void* base, int64_t i) {
  const unsigned short b = __ldg(static_cast<const unsigned short*>(base) + i);
  return __uint_as_float(((uint32_t)b) << 16);
}

}  // namespace q3s
