// q8k.cuh -- Q8_K activation quantization on sm_100a.
//
// One warp per 256-value block.  Lane l owns values 8l..8l+7.  The block
// maximum is the FIRST value of largest magnitude (strict '>' in index
// order), iscale = -127/max and scale = 1/iscale are IEEE divisions, and
// codes are ties-to-even roundings of the rounded binary32 product, clamped
// above at 127: the Source contract of reference src/kernels.rs:463-522.
// With `pinned`, codes follow the fused round of src/kernels.rs:421-428.
#pragma once

#include "common.cuh"

namespace prism {

constexpr int kQ8KBytes = 292;  // f32 scale, 256 x i8, 16 x i16

// Quantize one block held 8-per-lane in v[].  Outputs the block scale, this
// lane's 8 codes and the sum of the 16-value group this lane shares with
// lane^1.  Returns status bits (nonfinite input, range violation).
__device__ __forceinline__ unsigned q8k_quantize_regs(const float (&v)[8], int lane,
                                                      bool pinned, float &scale,
                                                      int8_t (&q)[8], int &pair_sum) {
  unsigned st = 0;
  float best = 0.0f;
  int best_idx = 0x7fffffff;
  bool finite = true;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    finite &= is_finite_f(v[i]);
    if (fabsf(v[i]) > fabsf(best)) {
      best = v[i];
      best_idx = lane * 8 + i;
    }
  }
  // larger magnitude wins, ties go to the smaller index
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    float ob = __shfl_xor_sync(0xffffffffu, best, off);
    int oi = __shfl_xor_sync(0xffffffffu, best_idx, off);
    float a = fabsf(best), b = fabsf(ob);
    if (b > a || (b == a && oi < best_idx)) {
      best = ob;
      best_idx = oi;
    }
  }
  finite = __all_sync(0xffffffffu, finite);
  if (!finite) st |= kStatusNonfinite;
  const float maximum = best;  // +0.0 when every value is zero
  scale = 0.0f;
  if (maximum == 0.0f || !finite) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = 0;
  } else {
    const float iscale = __fdiv_rn(-127.0f, maximum);
    if (!is_finite_f(iscale)) {
      st |= kStatusInvalid;
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
      scale = __fdiv_rn(1.0f, iscale);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int qi;
        if (pinned) {
          float r = __fmaf_rn(iscale, v[i], 12582912.0f);
          qi = (int)(__float_as_uint(r) & 0x007fffffu) - 0x00400000;
          qi = min(qi, 127);
          if (qi < -128) {
            st |= kStatusInvalid;
            qi = 0;
          }
        } else {
          float r = fminf(rintf(__fmul_rn(v[i], iscale)), 127.0f);
          if (!(r >= -127.0f && r <= 127.0f)) {
            st |= kStatusInvalid;
            r = 0.0f;
          }
          qi = (int)r;
        }
        q[i] = (int8_t)qi;
      }
    }
  }
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += q[i];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  pair_sum = s;
  return st;
}

// Quantize one block held 8-per-lane and write the AoS block at `out`
// (4-byte aligned).  Returns status bits.
__device__ __forceinline__ unsigned q8k_block_from_regs(const float (&v)[8], int lane,
                                                        bool pinned, uint8_t *out) {
  float scale;
  int8_t q[8];
  int s;
  const unsigned st = q8k_quantize_regs(v, lane, pinned, scale, q, s);
  if (lane == 0) *reinterpret_cast<float *>(out) = scale;
  uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) |
                ((uint32_t)(uint8_t)q[2] << 16) | ((uint32_t)(uint8_t)q[3] << 24);
  uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) |
                ((uint32_t)(uint8_t)q[6] << 16) | ((uint32_t)(uint8_t)q[7] << 24);
  uint32_t *vw = reinterpret_cast<uint32_t *>(out + 4);
  vw[lane * 2] = w0;
  vw[lane * 2 + 1] = w1;
  if ((lane & 1) == 0) reinterpret_cast<int16_t *>(out + 260)[lane >> 1] = (int16_t)s;
  return st;
}

// x: n floats (n = 256 * nblocks), 16-byte aligned.  out: nblocks AoS blocks.
__global__ void __launch_bounds__(256) q8k_quantize_kernel(const float *__restrict__ x,
                                                           int nblocks, int pinned,
                                                           uint8_t *__restrict__ out,
                                                           unsigned *status) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  grid_dependency_wait();  // x may be the previous kernel's output
  grid_dependents_launch();
  if (warp >= nblocks) return;
  const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)warp * 256 + lane * 8);
  float4 a = src[0], b = src[1];
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  unsigned st = q8k_block_from_regs(v, lane, pinned != 0, out + (size_t)warp * kQ8KBytes);
  if (st && lane == 0) report(status, st);
}

}  // namespace prism
