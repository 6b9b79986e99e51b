// common.cuh -- shared device helpers for the sm_100a kernels.
//
// Status word: every kernel reports failures by OR-ing a bit into a
// device-resident status word that the host reads after the work it
// enqueued (no __trap, no device assert).  Every spin-wait is bounded.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace prism {

// Status bits (device side).  Host maps them to PRISM_B200_E_* codes.
enum : unsigned {
  kStatusNonfinite = 1u << 0,  // nonfinite activation scale or output
  kStatusInvalid = 1u << 1,    // quantizer range violation
  kStatusTimeout = 1u << 2,    // a bounded wait expired
};

// Upper bound on any device-side wait, in nanoseconds of %globaltimer: far
// above any legitimate latency, short enough that a lost completion ends the
// kernel with a status bit instead of hanging the GPU.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report(unsigned *status, unsigned bit) {
  atomicOr(status, bit);
}

// Optional kernel timelines (globaltimer ns): CTA 0 stamps its progress
// points; on exit every CTA raises slot 7 to its exit time, so slot 7 ends
// as the last CTA's exit.
__device__ __forceinline__ void trace_stamp(unsigned long long *trace, int slot) {
  if (trace && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
    trace[slot] = global_timer_ns();
}
__device__ __forceinline__ void trace_exit(unsigned long long *trace) {
  if (trace && threadIdx.x == 0) {
    const unsigned long long t = global_timer_ns();
    if (blockIdx.x == 0 && blockIdx.y == 0) trace[6] = t;
    atomicMax(&trace[7], t);
  }
}

// ---- binary16 <-> binary32 --------------------------------------------------
// The hardware conversions: widening is exact for every binary16 value
// (subnormals included), narrowing rounds to nearest even with overflow to
// infinity -- the IEEE conversions the reference's half crate performs.
// Results differ from a bit-level restatement only in NaN payloads, which
// no valid input carries (scales are checked finite at upload).

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}

__device__ __forceinline__ uint16_t float_to_half_bits(float f) {
  uint16_t h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return h;
}

__device__ __forceinline__ float round_f16(float f) {
  return half_bits_to_float(float_to_half_bits(f));
}

__device__ __forceinline__ bool is_finite_f(float v) {
  return (__float_as_uint(v) & 0x7f800000u) != 0x7f800000u;
}

// binary32 transcendentals evaluated in binary64 and rounded once: the
// correctly rounded result for all but vanishingly rare inputs.  The
// reference's host libm (expf/logf/sinf/cosf evaluated in binary64
// internally) returns the same values, so activations feeding the Q8_K
// quantizer agree bit for bit instead of differing by an ulp, which the
// quantizer would otherwise amplify into whole-code flips.
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log_cr(float x) { return (float)log((double)x); }
__device__ __forceinline__ float sin_cr(float x) { return (float)sin((double)x); }
__device__ __forceinline__ float cos_cr(float x) { return (float)cos((double)x); }

// reference src/kernels.rs:3365-3368: silu(v) = v / (1 + exp(-v))
__device__ __forceinline__ float silu_f(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, exp_cr(-v)));
}

// ---- byte dot products -----------------------------------------------------

// sum of 4 (unsigned byte of a) * (signed byte of b) + c
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---- mbarrier + bulk async copy (sm_90+ PTX) -------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared accesses before later
// async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> shared, completing `bytes` of transaction on bar.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], "
      "%2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of the phase's completion.
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; returns false (and reports) if the phase never completed.
// A phase that already completed is seen by a non-blocking test.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, unsigned parity,
                                                  unsigned *status) {
  if (mbar_test_wait(bar, parity) || mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report(status, kStatusTimeout);
      return false;
    }
  }
  return true;
}

// ---- programmatic dependent launch -----------------------------------------
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace prism
