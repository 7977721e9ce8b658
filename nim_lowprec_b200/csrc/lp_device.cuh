// lp_device.cuh -- sm_100a device helpers shared by the lowprec kernels:
// mbarrier + 1-D bulk-copy (TMA) staging, packed f32x2 arithmetic, mixed-sign
// dp4a, byte permutes, and the bounded-wait / error-flag discipline.
//
// Floating-point policy (the GPU analogue of the reference's
// -ffp-contract=off, simd/dequant.nim:36): every multiply and add on a
// bit-exact path is an explicit round-to-nearest PTX op (mul.rn / add.rn /
// their f32x2 forms, or __fmul_rn/__fadd_rn) so nvcc can never contract a
// multiply feeding an add into an FMA.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "lowprec_cuda.h"

namespace lp {

// ----------------------------------------------------------------- errors
// Device-side failures never trap: a wait that runs out sets this word (and
// the kernel unwinds), the host reads it with lp_device_error().  The build
// is not relocatable-device-code, so each translation unit with waiting
// kernels has its own word and exports a host accessor (take_error_*).
static __device__ unsigned int g_device_error = 0;

__device__ __forceinline__ void raise_error(unsigned int code) {
  atomicCAS(&g_device_error, 0u, code);
}

// Every spin on an mbarrier gives up after this many nanoseconds (global
// timer) and reports LP_ERR_TIMEOUT.  Kernels here run for microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------- mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)),
               "r"(bytes)
               : "memory");
}
// try_wait may suspend the thread until the phase completes or the hint
// (ns) runs out, so a waiting warp does not spin on the issue slots the
// working warps of its SM sub-partition need.
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, "
      "0, p; }"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Bounded wait: true on success; false on timeout (error word set) or when
// another warp of the CTA has already given up (`abort` non-zero), so one
// failure unwinds the whole CTA within one time limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      raise_error(LP_ERR_TIMEOUT);
      if (abort) *abort = 1;
      return false;
    }
  }
}

// Bounded wait for warps whose wait is not on the critical path (a producer
// waiting for a free stage, a folder waiting for a finished tile): between
// polls the thread sleeps 32..256 ns, so a waiting warp leaves the issue
// slots of its sub-partition to the warps doing the work.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity,
                                               volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  uint32_t ns = 32;
  while (true) {
    __nanosleep(ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      raise_error(LP_ERR_TIMEOUT);
      if (abort) *abort = 1;
      return false;
    }
    if (ns < 256) ns <<= 1;
  }
}

// ----------------------------------------------------- bulk (TMA) copies
// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(bar)), "l"(policy)
      : "memory");
}
// L2 policy for a one-pass weight stream: evict first.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------- f32x2 (packed)
__device__ __forceinline__ uint64_t pk(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Rounded packed product a*b computed as fma(a, b, z) with z = -0.0 supplied
// at run time (a kernel parameter).  fma(a, b, -0) is exactly round(a*b),
// signed zeros included, and because the compiler cannot see that z is zero
// it cannot merge this product with the add that consumes it -- it does
// merge mul.rn.f32x2 into a following add.rn.f32x2 (measured on sm_100a),
// which would turn the reference's two roundings into one.
__device__ __forceinline__ uint64_t mul2_rn(uint64_t a, uint64_t b, uint64_t z) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(z));
  return d;
}
__device__ __forceinline__ float fmul(float a, float b) {
  float d;
  asm("mul.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float fadd(float a, float b) {
  float d;
  asm("add.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// --------------------------------------------------------- int helpers
// a: four unsigned bytes, b: four signed bytes, exact int32 dot + c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// a: four unsigned bytes, b: four unsigned bytes.
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// a: four signed bytes, b: four unsigned bytes.
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// int32 -> fp32, round to nearest even (same as C's conversion of an int32).
__device__ __forceinline__ float i2f_rn(int v) { return __int2float_rn(v); }

// fp16 bits -> fp32 (exact).
__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// ------------------------------------------------------------ math ---
__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace lp
