// peak.cuh -- the dense int8 tensor-core rate of this device, measured.
//
// One CTA per SM issues back-to-back tcgen05.mma.kind::i8 (M = 128, N = 256,
// K = 32, s32 accumulators in tensor memory) from operands resident in shared
// memory: no global traffic, nothing but the tensor pipe.  The rate it
// reaches is the denominator the GEMM's tensor roofline is quoted against.
#pragma once

#include "gemm.cuh"

namespace prism {

constexpr int kPeakM = 128, kPeakN = 256, kPeakK = 32;

__global__ void __launch_bounds__(128) tensor_peak_i8_kernel(int iters, unsigned *status) {
  __shared__ __align__(1024) uint8_t a[kPeakM * kPeakK];
  __shared__ __align__(1024) uint8_t b[kPeakN * kPeakK];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5;
  // any operand values serve; zeros keep the accumulators from overflowing
  for (int i = tid; i < kPeakM * kPeakK / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(a)[i] = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < kPeakN * kPeakK / 16; i += blockDim.x)
    reinterpret_cast<uint4 *>(b)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (warp == 0) {
    tmem_alloc(&tbase, kPeakN);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init_fence();
  }
  fence_proxy_async_smem();  // generic stores -> tensor-core reads
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t d = tbase;
  if (tid == 0) {
    // K-major, no swizzle: K-adjacent 16-byte core columns rows*16 bytes
    // apart, 8-row core matrices 128 bytes apart
    const uint64_t ad = umma_smem_desc(smem_addr(a), kPeakM * 16, 128);
    const uint64_t bd = umma_smem_desc(smem_addr(b), kPeakN * 16, 128);
    constexpr uint32_t idesc = umma_idesc_i8(kPeakM, kPeakN);
    for (int i = 0; i < iters; ++i) umma_i8(d, ad, bd, idesc, i > 0 ? 1u : 0u);
    umma_commit(&bar);
    mbar_wait_bounded(&bar, 0u, status);  // a timeout is reported in the status word
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(d, kPeakN);
}

}  // namespace prism
