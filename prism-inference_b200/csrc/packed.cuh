// packed.cuh -- the reference's own packed ternary formats, PQ2 (type 142)
// and PTQ1 (type 143), projected on the device.
//
// PQ2 holds 128 weights in 34 bytes: a binary16 scale, then 32 bytes of
// 2-bit codes, weight 4j + k in bits 2k..2k+1 of byte j, value code - 1 (code
// 3 is the native decoder's +2; reference src/kernels.rs:178-180).  PTQ1
// holds the same weights in 28 bytes: 26 bytes of base-3 fractional digits
// (byte b stands for the digits of b / 256: five per byte for weights 0-119,
// four for weights 120-127; reference tools/ternary/src/lib.rs:193-250) and
// the binary16 scale last.  Weights stay on the device as uploaded.
//
// Activation contract (reference src/kernels.rs:1663-1674): PQ2 with a
// multiple of 256 columns takes Q8_K blocks -- per PQ2 block i, d = scale_i *
// act[i / 2].scale and the exact integer dot with that block's half, output
// = output + d * dot (fma when fused), blocks in order (src/kernels.rs:941-
// 959); PTQ1, and PQ2 otherwise, take Q8_0 blocks -- per block, sum over its
// four 32-weight groups of act.scale * dot in binary32, output = output + d *
// sum (src/kernels.rs:1043-1063).
//
// One warp per row: lane l decodes block l of each round of 32 blocks into a
// 128-byte shared-memory slot and forms that block's (d, s) pair; the row's
// chain then runs over the round in block order on every lane through
// shuffles, so the binary32 sums keep the reference's order.
#pragma once

#include "common.cuh"

namespace prism {

constexpr int kPackedWarps = 8;  // rows per CTA

// Q8_0 activation block of the C ABI (the reference's Q8Block: scale and
// code sum as binary32, 32 codes).
struct Q8Act {
  float scale, sum;
  int8_t values[32];
};
static_assert(sizeof(Q8Act) == 40, "Q8_0 activation block");

__host__ __device__ constexpr int pq_block_bytes(uint32_t kind) {
  return kind == 142 ? 34 : kind == 143 ? 28 : 0;
}

// digit d (0..4) of byte b's base-3 expansion of b / 256 at bits 2d..2d+1
__device__ __forceinline__ uint32_t ptq_digits(uint32_t b) {
  uint32_t out = 0, f = b;
#pragma unroll
  for (int d = 0; d < 5; ++d) {
    f *= 3u;
    out |= (f >> 8) << (2 * d);
    f &= 255u;
  }
  return out;
}

// The 128 weights (-1..2) of one block into w[128].
__device__ __forceinline__ void packed_decode(uint32_t kind, const uint8_t *blk, int8_t *w) {
  if (kind == 142) {
    for (int j = 0; j < 32; ++j) {
      const uint32_t c = blk[2 + j];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[4 * j + k] = (int8_t)(((c >> (2 * k)) & 3u) - 1);
    }
  } else {
    for (int m = 0; m < 16; ++m) {
      const uint32_t dg = ptq_digits(blk[m]);
#pragma unroll
      for (int d = 0; d < 5; ++d) w[m + 16 * d] = (int8_t)(((dg >> (2 * d)) & 3u) - 1);
    }
    for (int m = 0; m < 8; ++m) {
      const uint32_t dg = ptq_digits(blk[16 + m]);
#pragma unroll
      for (int d = 0; d < 5; ++d) w[80 + m + 8 * d] = (int8_t)(((dg >> (2 * d)) & 3u) - 1);
    }
    for (int h = 0; h < 2; ++h) {
      const uint32_t dg = ptq_digits(blk[24 + h]);
#pragma unroll
      for (int d = 0; d < 4; ++d) w[120 + h + 2 * d] = (int8_t)(((dg >> (2 * d)) & 3u) - 1);
    }
  }
}

__device__ __forceinline__ int packed_idot(const int8_t *w, const int8_t *a, int n) {
  int s = 0;
  for (int i = 0; i < n; ++i) s += (int)w[i] * (int)a[i];
  return s;
}

struct PackedArgs {
  const uint8_t *w;   // rows x nb blocks, row-major
  uint32_t kind;
  long rows;
  int nb;             // blocks of 128 weights per row
  const void *act;    // Q8_K blocks (292 B) when q8k, else Q8Act blocks
  int q8k, fused;
  float *y;
  unsigned *status;
};

__global__ void __launch_bounds__(kPackedWarps * 32) packed_matvec_kernel(PackedArgs a) {
  // a lane's decoded block: 128 weights, slots 132 bytes apart so that the
  // lanes' bytes at one offset fall in distinct banks
  __shared__ __align__(16) int8_t dec[kPackedWarps][32][132];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * kPackedWarps + warp;
  grid_dependency_wait();
  grid_dependents_launch();
  if (row >= a.rows) return;
  const int bb = pq_block_bytes(a.kind);
  const uint8_t *rw = a.w + (size_t)row * a.nb * bb;
  int8_t *w = dec[warp][lane];
  float output = 0.0f;
  bool bad_scale = false;
  for (int r0 = 0; r0 < a.nb; r0 += 32) {
    const int b = r0 + lane, count = min(32, a.nb - r0);
    float d = 0.0f, s = 0.0f;
    if (b < a.nb) {
      const uint8_t *blk = rw + (size_t)b * bb;
      const uint8_t *sp = a.kind == 142 ? blk : blk + 26;
      const float scale = half_bits_to_float((uint16_t)(sp[0] | (sp[1] << 8)));
      bad_scale |= !is_finite_f(scale);
      packed_decode(a.kind, blk, w);
      if (a.q8k) {
        const uint8_t *ab = static_cast<const uint8_t *>(a.act) + (size_t)(b / 2) * 292;
        const float as = *reinterpret_cast<const float *>(ab);
        d = __fmul_rn(scale, as);
        s = (float)packed_idot(w, reinterpret_cast<const int8_t *>(ab + 4) + (b % 2) * 128, 128);
      } else {
        const Q8Act *g = static_cast<const Q8Act *>(a.act) + (size_t)b * 4;
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          sum = __fadd_rn(sum, __fmul_rn(g[q].scale, (float)packed_idot(w + 32 * q, g[q].values, 32)));
        d = scale;
        s = sum;
      }
    }
    // the row's chain over this round's blocks, in block order
    for (int j = 0; j < count; ++j) {
      const float dj = __shfl_sync(0xffffffffu, d, j), sj = __shfl_sync(0xffffffffu, s, j);
      output = a.q8k && a.fused ? fmaf(dj, sj, output) : __fadd_rn(output, __fmul_rn(dj, sj));
    }
  }
  bad_scale = __any_sync(0xffffffffu, bad_scale);
  if (lane == 0) {
    if (bad_scale || !is_finite_f(output)) report(a.status, kStatusNonfinite);
    a.y[row] = output;
  }
}

// Q8_0 activations of n values (reference src/kernels.rs:552-617 without the
// pinned or native-scale options): per 32-value block, d = max|x| / 127, the
// stored scale round_f16(d), codes round-half-away(x * (1 / d)) (0 when d is
// 0), sum round_f16(code sum * d).  One warp per block, a value per lane.
__global__ void __launch_bounds__(256) q8_0_quantize_kernel(const float *x, long nblocks,
                                                            Q8Act *out, unsigned *status) {
  const long blk = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  grid_dependency_wait();
  grid_dependents_launch();
  if (blk >= nblocks) return;
  const float v = x[blk * 32 + lane];
  const bool finite = __all_sync(0xffffffffu, is_finite_f(v));
  float m = fabsf(v);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const float d = __fdiv_rn(m, 127.0f);
  const float inv = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  const float scale = round_f16(d);
  const float r = roundf(__fmul_rn(v, inv));
  const bool in_range = __all_sync(0xffffffffu, r >= -127.0f && r <= 127.0f);
  const int q = in_range ? (int)r : 0;
  int sum = q;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  Q8Act &o = out[blk];
  o.values[lane] = (int8_t)q;
  if (lane == 0) {
    o.scale = scale;
    o.sum = round_f16(__fmul_rn((float)sum, d));
    if (!finite || !is_finite_f(scale)) report(status, kStatusNonfinite);
    else if (!in_range) report(status, kStatusInvalid);
  }
}

}  // namespace prism
