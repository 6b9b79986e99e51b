// kquant.cuh -- the remaining kinds of the reference's Q8_K activation
// contract on the device: TQ1_0 (34) and Q3_K, Q4_K, Q5_K, Q6_K (11-14)
// (reference src/kernels.rs:1653-1674 ActivationContract::for_tensor).
// Weights stay on the device as uploaded (the reference's block bytes).
//
// Per 256-weight block against one Q8_K activation block:
//   - TQ1_0 (54 B): 48 bytes of five base-3 digits and 4 of four, fp16 d at
//     52; the exact integer sum; row: sum += (f32)int * (d * s), blocks in
//     order (reference src/kernels/tquants.rs:148-188, 270-287);
//   - Q3_K (110 B), Q4_K (144 B), Q5_K (176 B), Q6_K (210 B): eight exact
//     integer lane sums (element i into lane i % 8, weighted by its group's
//     scale) and, for Q4_K/Q5_K, the minimum sum over the activation's group
//     sums; row: lane[l] += (d * s) * (f32)int[l], Q4_K/Q5_K also
//     sum -= (dmin * s) * (f32)msum, blocks in order, then sum += lane[0..7]
//     in order (reference src/kernels/kquants.rs:53-130, 202-420).
// The integer parts are exact, so any summation order gives them; every
// binary32 operation keeps the reference's order.
//
// One warp per row: lane l forms block l of each round of 32 blocks, and the
// row's binary32 chain runs over the round in block order on every lane
// through shuffles.  Correctness-first: these kinds are on no benchmarked
// path.
#pragma once

#include "common.cuh"

namespace prism {

constexpr int kKqWarps = 8;  // rows per CTA

__host__ __device__ constexpr int kquant_block_bytes(uint32_t kind) {
  return kind == 34 ? 54 : kind == 11 ? 110 : kind == 12 ? 144 : kind == 13 ? 176
                                                                            : kind == 14 ? 210 : 0;
}

__device__ __forceinline__ float kq_half(const uint8_t *p) {
  return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// TQ1_0 digit e of byte b: (3 * ((b * 3^e) mod 256)) / 256 - 1.
__device__ __forceinline__ int tq1_digit(uint32_t b, int e) {
  const uint32_t p = e == 0 ? 1u : e == 1 ? 3u : e == 2 ? 9u : e == 3 ? 27u : 81u;
  return (int)(((b * p) & 255u) * 3u / 256u) - 1;
}

// TQ1_0 weight i of a block (element order of the reference's codes()).
__device__ __forceinline__ int tq1_value(const uint8_t *blk, int i) {
  if (i < 160) return tq1_digit(blk[i % 32], i / 32);
  if (i < 240) return tq1_digit(blk[32 + (i - 160) % 16], (i - 160) / 16);
  return tq1_digit(blk[48 + (i - 240) % 4], (i - 240) / 4);
}

// Q4_K / Q5_K 6-bit group scale and minimum from the 12 packed bytes.
__device__ __forceinline__ void q45_scale_min(int g, const uint8_t *s, int &sc, int &mn) {
  if (g < 4) {
    sc = s[g] & 63;
    mn = s[g + 4] & 63;
  } else {
    sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
    mn = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
  }
}

// Weight i (integer) and its group's scale of a K-quant block.
__device__ __forceinline__ int kq_value(uint32_t kind, const uint8_t *b, int i) {
  switch (kind) {
    case 11: {
      const int low = (b[32 + i / 128 * 32 + i % 32] >> (2 * (i % 128 / 32))) & 3;
      return low - ((b[i % 32] & (1 << (i / 32))) ? 0 : 4);
    }
    case 12: return (b[16 + i / 64 * 32 + i % 32] >> (4 * (i % 64 / 32))) & 15;
    case 13: {
      const int v = (b[48 + i / 64 * 32 + i % 32] >> (4 * (i % 64 / 32))) & 15;
      return v + ((b[16 + i % 32] & (1 << (i / 32))) ? 16 : 0);
    }
    default: {  // 14
      const int part = i % 128 / 32;
      const int low = (b[i / 128 * 64 + part % 2 * 32 + i % 32] >> (4 * (part / 2))) & 15;
      const int high = (b[128 + i / 128 * 32 + i % 32] >> (2 * part)) & 3;
      return (low | (high << 4)) - 32;
    }
  }
}

__device__ __forceinline__ int kq_group_scale(uint32_t kind, const uint8_t *b, int g) {
  if (kind == 11)
    return (int)(((b[96 + g % 8] >> (4 * (g / 8))) & 15) |
                 (((b[104 + g % 4] >> (2 * (g / 4))) & 3) << 4)) -
           32;
  if (kind == 14) return (int)(int8_t)b[192 + g];
  int sc, mn;
  q45_scale_min(g, b + 4, sc, mn);
  return sc;
}

struct KquantArgs {
  const uint8_t *w;   // rows x nb blocks, row-major, as uploaded
  uint32_t kind;
  long rows;
  int nb;             // 256-weight blocks per row
  const uint8_t *act; // Q8_K blocks, 292 B each
  float *y;
  unsigned *status;
};

__global__ void __launch_bounds__(kKqWarps * 32) kquant_matvec_kernel(KquantArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * kKqWarps + warp;
  grid_dependency_wait();
  grid_dependents_launch();
  if (row >= a.rows) return;
  const int bb = kquant_block_bytes(a.kind);
  const uint8_t *rw = a.w + (size_t)row * a.nb * bb;
  float sum = 0.0f, lanes[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) lanes[l] = 0.0f;
  bool bad = false;
  for (int r0 = 0; r0 < a.nb; r0 += 32) {
    const int b = r0 + lane, count = min(32, a.nb - r0);
    int ints[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int msum = 0;
    float d = 0.0f, dmin = 0.0f, s = 0.0f;
    if (b < a.nb) {
      const uint8_t *blk = rw + (size_t)b * bb;
      const uint8_t *ab = a.act + (size_t)b * 292;
      const int8_t *q = reinterpret_cast<const int8_t *>(ab + 4);
      const int16_t *sums = reinterpret_cast<const int16_t *>(ab + 260);
      s = *reinterpret_cast<const float *>(ab);
      if (a.kind == 34) {
        d = kq_half(blk + 52);
        for (int i = 0; i < 256; ++i) ints[0] += tq1_value(blk, i) * (int)q[i];
      } else {
        const int group = (a.kind == 12 || a.kind == 13) ? 32 : 16;
        d = kq_half(a.kind == 11 ? blk + 108 : a.kind == 14 ? blk + 208 : blk);
        if (a.kind == 12 || a.kind == 13) dmin = kq_half(blk + 2);
        for (int g = 0; g < 256 / group; ++g) {
          const int sc = kq_group_scale(a.kind, blk, g);
          for (int j = 0; j < group; ++j) {
            const int i = g * group + j;
            ints[i & 7] += sc * kq_value(a.kind, blk, i) * (int)q[i];
          }
          if (a.kind == 12 || a.kind == 13) {
            int sc2, mn;
            q45_scale_min(g, blk + 4, sc2, mn);
            msum += ((int)sums[2 * g] + (int)sums[2 * g + 1]) * mn;
          }
        }
      }
      bad |= !is_finite_f(d) || !is_finite_f(dmin) || !is_finite_f(s);
    }
    // the row's chain over this round's blocks, in block order
    for (int j = 0; j < count; ++j) {
      const float dj = __shfl_sync(0xffffffffu, d, j), sj = __shfl_sync(0xffffffffu, s, j);
      if (a.kind == 34) {
        const int ij = __shfl_sync(0xffffffffu, ints[0], j);
        sum = __fadd_rn(sum, __fmul_rn((float)ij, __fmul_rn(dj, sj)));
        continue;
      }
      const float dact = __fmul_rn(dj, sj);
#pragma unroll
      for (int l = 0; l < 8; ++l)
        lanes[l] =
            __fadd_rn(lanes[l], __fmul_rn(dact, (float)__shfl_sync(0xffffffffu, ints[l], j)));
      if (a.kind == 12 || a.kind == 13) {
        const float mj = __shfl_sync(0xffffffffu, dmin, j);
        const int msj = __shfl_sync(0xffffffffu, msum, j);
        sum = __fsub_rn(sum, __fmul_rn(__fmul_rn(mj, sj), (float)msj));
      }
    }
  }
  if (a.kind != 34)
#pragma unroll
    for (int l = 0; l < 8; ++l) sum = __fadd_rn(sum, lanes[l]);
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    if (bad || !is_finite_f(sum)) report(a.status, kStatusNonfinite);
    a.y[row] = sum;
  }
}

// f32 rows -> TQ1_0 (34) or TQ2_0 (35) blocks (reference
// src/kernels/tquants.rs:288-336 quantize): d = max |x| stored as binary16;
// level = round-half-away(x * (1 / d)) + 1 (0 when d is 0); TQ2_0 ORs the
// levels into 2-bit fields, TQ1_0 folds five (or four, then times 3) levels
// per byte in base 3 and stores ceil(code * 256 / 243).  One CTA of 256
// threads per block, a thread per weight; the caller has checked nothing, so
// a nonfinite input reports invalid and an overflowing d nonfinite (the
// block is then left unwritten).
__global__ void __launch_bounds__(256) tq_quantize_kernel(uint32_t kind, const float *x,
                                                           uint8_t *out, unsigned *status) {
  __shared__ uint8_t level[256];
  __shared__ float red[8];
  const int i = threadIdx.x;
  const long b = blockIdx.x;
  grid_dependency_wait();
  grid_dependents_launch();
  const float v = x[b * 256 + i];
  if (!__syncthreads_and(is_finite_f(v))) {
    if (i == 0) report(status, kStatusInvalid);
    return;
  }
  float m = fabsf(v);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((i & 31) == 0) red[i >> 5] = m;
  __syncthreads();
  float d = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) d = fmaxf(d, red[w]);
  const uint16_t bits = float_to_half_bits(d);
  const float inverse = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  if (!is_finite_f(half_bits_to_float(bits)) || !is_finite_f(inverse)) {
    if (i == 0) report(status, kStatusNonfinite);
    return;
  }
  level[i] = (uint8_t)((int)roundf(__fmul_rn(v, inverse)) + 1);
  __syncthreads();
  const int size = kind == 35 ? 66 : 54;
  uint8_t *o = out + b * size;
  if (kind == 35) {
    if (i < 64) {
      const int half = i / 32, col = i % 32;
      unsigned byte = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) byte |= (unsigned)level[half * 128 + col + 32 * k] << (2 * k);
      o[i] = (uint8_t)byte;
    }
  } else if (i < 52) {
    const int first = i < 32 ? i : i < 48 ? 160 + i - 32 : 240 + i - 48;
    const int stride = i < 32 ? 32 : i < 48 ? 16 : 4, count = i < 48 ? 5 : 4;
    unsigned code = 0;
    for (int k = 0; k < count; ++k) code = code * 3 + level[first + k * stride];
    if (count == 4) code *= 3;
    o[i] = (uint8_t)((code * 256 + 242) / 243);
  }
  if (i == 0) {
    o[size - 2] = (uint8_t)(bits & 0xff);
    o[size - 1] = (uint8_t)(bits >> 8);
  }
}

}  // namespace prism
