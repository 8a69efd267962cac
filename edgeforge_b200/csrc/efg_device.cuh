// efg_device.cuh - device-side building blocks shared by the EdgeForge-B200 kernels:
// exact fp16/bf16 conversions, mbarrier + 1-D bulk-copy (TMA) wrappers with bounded
// waits, programmatic-dependent-launch hooks and warp reductions. sm_100a only.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "efg_status.h"

#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ < 1000
#error "EdgeForge-B200 kernels target sm_100a only"
#endif

namespace efg {

// ---------------------------------------------------------------- fp16 / bf16
// Exact binary16 -> binary32, the arithmetic of include/ef/fp16.h:44-66 in the
// reference (subnormals, inf and NaN payloads kept). The hardware conversion gives the
// same value for every non-NaN pattern; the bit-level form keeps NaN payloads too.
__device__ __forceinline__ float fp16_to_f32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  if (e == 0) return __uint_as_float(__float_as_uint(__uint2float_rn(m) * 5.9604644775390625e-08f) | sign);
  if (e == 31) return __uint_as_float(sign | 0x7F800000u | (m << 13));
  return __uint_as_float(sign | ((e + 112u) << 23) | (m << 13));
}

// binary32 -> binary16, round to nearest even; |x| >= 65520 -> inf; NaN -> quiet NaN
// keeping the top payload bits (include/ef/fp16.h:69-92). Integer arithmetic only.
__device__ __forceinline__ uint32_t f32_to_fp16(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return sign | 0x7E00u | ((a >> 13) & 0x3FFu);
  if (a >= 0x477FF000u) return sign | 0x7C00u;
  if (a < 0x38800000u) {
    if (a <= 0x33000000u) return sign;  // at or below 2^-25: rounds to zero
    const uint32_t e = a >> 23;         // 102..112
    const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    const uint32_t sh = 126u - e;       // 14..24
    uint32_t r = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return sign | r;
  }
  const uint32_t x = a - 0x38000000u;
  uint32_t r = x >> 13;
  const uint32_t dropped = x & 0x1FFFu;
  if (dropped > 0x1000u || (dropped == 0x1000u && (r & 1u))) ++r;
  return sign | r;
}

__device__ __forceinline__ float fp16_round(float f) { return fp16_to_f32(f32_to_fp16(f)); }

__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// ---------------------------------------------------------------- timing / errors
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every bounded wait gives up after this long and records EFG_ETIMEOUT. Normal waits
// in these kernels last microseconds.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ bool error_raised(const int* err) {
  return err && *reinterpret_cast<const volatile int*>(err) != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up (returns false and
// records EFG_ETIMEOUT in *err) after kWaitTimeoutNs, or as soon as another thread of
// the grid has recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
#pragma unroll 1
  for (int i = 0; i < 32; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u) {
      if (error_raised(err)) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        record_error(err, EFG_ETIMEOUT);
        return false;
      }
    }
  }
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps until it
// completes (or `ns` pass) instead of returning at once, so waiting warps leave the issue
// slots and pipes to the warps that work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// mbar_wait for warp-specialised kernels with many waiting warps: same bound and error
// behaviour, each poll sleeps up to 2 us on the barrier.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    if ((i & 7u) == 7u) {
      if (error_raised(err)) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        record_error(err, EFG_ETIMEOUT);
        return false;
      }
    }
  }
}

// SwiGLU element silu(g) * u of the reference (src/kernels.cpp:94-99), every rounding explicit
// so that the per-token, persistent and batched kernels that apply it give the same bits.
__device__ __forceinline__ float swiglu_value(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// ---------------------------------------------------------------- 1-D bulk copy (TMA)
// L2 policy for data read exactly once (weights streamed by a matvec).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 policy for data many CTAs read (activations shared by every output tile).
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> this CTA's shared memory, completion signalled on `bar` as tx bytes.
// dst, src and bytes must all be multiples of 16. The copy lands in this CTA only.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}

// 2-D TMA tensor load of one box (no multicast) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar,
                                            uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel may start before the previous kernel in the
// stream has finished; pdl_wait() blocks until it has and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Sums RB per-lane values over the 32 lanes at once (a reduce-scatter butterfly):
// afterwards lane L holds the total of row L / (32 / RB) in lanes where
// L % (32 / RB) == 0. Costs 2*RB-1 + log2(32/RB) shuffles instead of 5*RB.
template <int RB>
__device__ __forceinline__ float warp_reduce_rows(const float (&v)[RB], int lane) {
  if constexpr (RB == 1) {
    return warp_sum(v[0]);
  } else if constexpr (RB == 2) {
    const bool hi = lane & 16;
    float keep = hi ? v[1] : v[0];
    const float send = hi ? v[0] : v[1];
    keep += __shfl_xor_sync(0xFFFFFFFFu, send, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xFFFFFFFFu, keep, o);
    return keep;
  } else {
    static_assert(RB == 4, "RB must be 1, 2 or 4");
    const bool h16 = lane & 16;
    float k0 = h16 ? v[2] : v[0];
    float k1 = h16 ? v[3] : v[1];
    const float s0 = h16 ? v[0] : v[2];
    const float s1 = h16 ? v[1] : v[3];
    k0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 16);
    k1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 16);
    const bool h8 = lane & 8;
    float keep = h8 ? k1 : k0;
    const float send = h8 ? k0 : k1;
    keep += __shfl_xor_sync(0xFFFFFFFFu, send, 8);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) keep += __shfl_xor_sync(0xFFFFFFFFu, keep, o);
    return keep;
  }
}

}  // namespace efg
