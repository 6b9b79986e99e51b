// matvec.cuh -- batch-1 packed ternary / 2-bit projection on sm_100a.
//
// y[r] = sum_b term(r, b), where term is the reference's per-block binary32
// contribution and the sum is the reference's sequential binary32 chain over
// blocks (TQ2_0: reference src/kernels/tquants.rs:270-287; Q2_K:
// src/kernels/kquants.rs:346-420 kind 10).  Integer block dots are exact.
//
// Device weight layout ("tiled", built once at upload):
//   rows are grouped in 32-row tiles (the last tile zero padded); a UNIT is
//   one tile x one 256-column block, stored contiguously, units ordered
//   tile-major then block:
//     TQ2_0 unit (2112 B): qs[4 chunks][32 rows][16 B] | d[32 rows] fp16
//     Q2_K  unit (2688 B): qs[4][32][16 B] | scales[32][16 B] |
//                          d[32] fp16 | dmin[32] fp16
//   Chunk c of a row's block is bytes 16c..16c+15 of its 64 quant bytes.
//   The layout holds exactly the packed bytes (plus tile padding): HBM
//   traffic per projection equals the reference's packed size.
//
// Execution: each CTA owns a contiguous range of units, so its weight bytes
// are one contiguous HBM range, streamed by 1-D bulk async copies
// (cp.async.bulk) into per-warp shared-memory rings (kDepth slots per warp,
// mbarrier completion).  Lane l of a warp computes row 32t+l of the unit:
// weights are lane-private 16-byte chunks, activations are broadcast
// 16-byte shared loads, byte products use dp4a.  Each unit's 32 terms go to
// a scratch row [tile][block][32]; the warp that completes a tile (counter
// reaches nb) sums its terms in block order -- exactly the reference's
// chain -- and writes y.  The counter is reset by that warp for the next
// launch.
#pragma once

#include "common.cuh"
#include "q8k.cuh"

namespace prism {

constexpr int kTileRows = 32;
constexpr int kTq2Unit = 2112;
constexpr int kQ2kUnit = 2688;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kDepth = 4;

template <int KIND>
struct UnitTraits;
template <>
struct UnitTraits<35> {
  static constexpr int bytes = kTq2Unit;
};
template <>
struct UnitTraits<10> {
  static constexpr int bytes = kQ2kUnit;
};

// Shared-memory layout of the matvec kernel (dynamic smem).
struct MatvecSmem {
  static __host__ __device__ constexpr int act_values(int nb) { return 0; }
  static __host__ __device__ constexpr int act_scale(int nb) { return nb * 256; }
  static __host__ __device__ constexpr int act_sums(int nb) { return nb * 256 + nb * 4; }
  static __host__ __device__ constexpr int act_asum(int nb) { return nb * 256 + nb * 4 + nb * 32; }
  static __host__ __device__ constexpr int bars(int nb) {
    return ((nb * 256 + nb * 4 + nb * 32 + nb * 4) + 15) / 16 * 16;
  }
  static __host__ __device__ constexpr int slots(int nb) {
    return (bars(nb) + kWarps * kDepth * 8 + 127) / 128 * 128;
  }
  static __host__ __device__ constexpr int total(int nb, int unit_bytes) {
    return slots(nb) + kWarps * kDepth * unit_bytes;
  }
};

enum MatvecMode : int {
  kModeOutput = 0,  // y = W x
  kModeInts = 1,    // exact per-block integer dots to ints / ints2
};

struct MatvecArgs {
  const uint8_t *w;      // tiled units
  const uint8_t *act;    // nb AoS Q8_K blocks
  int nb;                // blocks per row
  int ntiles;            // 32-row tiles
  int rows;              // true rows
  float *y;              // rows floats (kModeOutput)
  float *partial;        // ntiles*nb*32 floats scratch
  unsigned *tile_cnt;    // ntiles counters, zero between launches
  int32_t *ints;         // rows*nb (kModeInts)
  int32_t *ints2;        // rows*nb (kModeInts, Q2_K min sums)
  unsigned *status;
};

// One unit's contribution for this lane's row: TQ2_0.
__device__ __forceinline__ void tq2_unit(const uint8_t *slot, const int8_t *av, int asum,
                                         float s, int lane, int &dot, float &term) {
  const uint4 *qs = reinterpret_cast<const uint4 *>(slot);
  int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 wq = qs[c * 32 + lane];
    const int8_t *base = av + (c >> 1) * 128 + (c & 1) * 16;
    int4 a0 = *reinterpret_cast<const int4 *>(base);
    int4 a1 = *reinterpret_cast<const int4 *>(base + 32);
    int4 a2 = *reinterpret_cast<const int4 *>(base + 64);
    int4 a3 = *reinterpret_cast<const int4 *>(base + 96);
    acc0 = dp4a_us(wq.x & 0x03030303u, a0.x, acc0);
    acc0 = dp4a_us(wq.y & 0x03030303u, a0.y, acc0);
    acc0 = dp4a_us(wq.z & 0x03030303u, a0.z, acc0);
    acc0 = dp4a_us(wq.w & 0x03030303u, a0.w, acc0);
    acc1 = dp4a_us(wq.x & 0x0c0c0c0cu, a1.x, acc1);
    acc1 = dp4a_us(wq.y & 0x0c0c0c0cu, a1.y, acc1);
    acc1 = dp4a_us(wq.z & 0x0c0c0c0cu, a1.z, acc1);
    acc1 = dp4a_us(wq.w & 0x0c0c0c0cu, a1.w, acc1);
    acc2 = dp4a_us(wq.x & 0x30303030u, a2.x, acc2);
    acc2 = dp4a_us(wq.y & 0x30303030u, a2.y, acc2);
    acc2 = dp4a_us(wq.z & 0x30303030u, a2.z, acc2);
    acc2 = dp4a_us(wq.w & 0x30303030u, a2.w, acc2);
    acc3 = dp4a_us(wq.x & 0xc0c0c0c0u, a3.x, acc3);
    acc3 = dp4a_us(wq.y & 0xc0c0c0c0u, a3.y, acc3);
    acc3 = dp4a_us(wq.z & 0xc0c0c0c0u, a3.z, acc3);
    acc3 = dp4a_us(wq.w & 0xc0c0c0c0u, a3.w, acc3);
  }
  // plane j products carry a factor 4^j; codes are weight+1, so subtract the
  // block's activation sum to obtain sum((code-1)*q) exactly.
  dot = acc0 + (acc1 >> 2) + (acc2 >> 4) + (acc3 >> 6) - asum;
  uint16_t dh = reinterpret_cast<const uint16_t *>(slot + 2048)[lane];
  float d = half_bits_to_float(dh);
  term = __fmul_rn((float)dot, __fmul_rn(d, s));
}

__device__ __forceinline__ unsigned byte_of(const uint4 &v, int g) {
  unsigned w = (g < 4) ? v.x : (g < 8) ? v.y : (g < 12) ? v.z : v.w;
  return (w >> (8 * (g & 3))) & 0xffu;
}

// One unit's contribution for this lane's row: Q2_K.
__device__ __forceinline__ void q2k_unit(const uint8_t *slot, const int8_t *av,
                                         const int16_t *asums, float s, int lane, int &isum,
                                         int &msum, float &term) {
  const uint4 *qs = reinterpret_cast<const uint4 *>(slot);
  uint4 sc = reinterpret_cast<const uint4 *>(slot + 2048)[lane];
  int is = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 wq = qs[c * 32 + lane];
    const int8_t *base = av + (c >> 1) * 128 + (c & 1) * 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const unsigned m = 0x03030303u << (2 * j);
      int4 a = *reinterpret_cast<const int4 *>(base + 32 * j);
      int acc = dp4a_us(wq.x & m, a.x, 0);
      acc = dp4a_us(wq.y & m, a.y, acc);
      acc = dp4a_us(wq.z & m, a.z, acc);
      acc = dp4a_us(wq.w & m, a.w, acc);
      const int g = 8 * (c >> 1) + 2 * j + (c & 1);
      is += (int)(byte_of(sc, g) & 15u) * (acc >> (2 * j));
    }
  }
  int ms = 0;
#pragma unroll
  for (int g = 0; g < 16; ++g) ms += (int)asums[g] * (int)(byte_of(sc, g) >> 4);
  isum = is;
  msum = ms;
  const uint16_t *dd = reinterpret_cast<const uint16_t *>(slot + 2048 + 512);
  float d = half_bits_to_float(dd[lane]);
  float dmin = half_bits_to_float(dd[32 + lane]);
  float t1 = __fmul_rn(__fmul_rn(s, d), (float)is);
  float t2 = __fmul_rn(__fmul_rn(s, dmin), (float)ms);
  term = __fsub_rn(t1, t2);
}

// Stage the Q8_K activation (AoS, 4-byte aligned) into shared memory as
// values[nb][256] | scale[nb] | sums[nb][16] | asum[nb].
__device__ __forceinline__ void stage_activation(const uint8_t *act, int nb, uint8_t *smem,
                                                 unsigned *status) {
  int8_t *values = reinterpret_cast<int8_t *>(smem + MatvecSmem::act_values(nb));
  float *scale = reinterpret_cast<float *>(smem + MatvecSmem::act_scale(nb));
  int16_t *sums = reinterpret_cast<int16_t *>(smem + MatvecSmem::act_sums(nb));
  int *asum = reinterpret_cast<int *>(smem + MatvecSmem::act_asum(nb));
  const uint32_t *src = reinterpret_cast<const uint32_t *>(act);
  // 73 words per block: word 0 scale, words 1..64 values, 65..72 sums
  for (int i = threadIdx.x; i < nb * 73; i += blockDim.x) {
    int b = i / 73, k = i % 73;
    uint32_t v = src[i];
    if (k == 0) {
      scale[b] = __uint_as_float(v);
    } else if (k <= 64) {
      reinterpret_cast<uint32_t *>(values)[b * 64 + (k - 1)] = v;
    } else {
      reinterpret_cast<uint32_t *>(sums)[b * 8 + (k - 65)] = v;
    }
  }
  __syncthreads();
  // per-block activation sums (from the codes), one warp per block
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < nb; b += blockDim.x >> 5) {
    const int32_t *vw = reinterpret_cast<const int32_t *>(values + b * 256);
    int s = __dp4a(vw[lane], 0x01010101, 0) + __dp4a(vw[lane + 32], 0x01010101, 0);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      asum[b] = s;
      if (!is_finite_f(scale[b])) report(status, kStatusNonfinite);
    }
  }
  __syncthreads();
}

template <int KIND, int MODE, bool PDL>
__global__ void __launch_bounds__(kThreads) matvec_kernel(MatvecArgs args) {
  constexpr int UNIT = UnitTraits<KIND>::bytes;
  extern __shared__ __align__(128) uint8_t smem[];
  const int nb = args.nb;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long total_units = (long)args.ntiles * nb;
  const long u0 = total_units * blockIdx.x / gridDim.x;
  const long u1 = total_units * (blockIdx.x + 1) / gridDim.x;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + MatvecSmem::bars(nb)) + warp * kDepth;
  uint8_t *slots = smem + MatvecSmem::slots(nb) + (size_t)warp * kDepth * UNIT;

  // Weights never depend on the previous kernel: start streaming them
  // before waiting on the grid dependency.
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < kDepth; ++k) mbar_init(&bars[k], 1);
    mbar_init_fence();
#pragma unroll
    for (int k = 0; k < kDepth; ++k) {
      long u = u0 + warp + (long)k * kWarps;
      if (u < u1) {
        mbar_arrive_expect_tx(&bars[k], UNIT);
        bulk_g2s(slots + k * UNIT, args.w + u * UNIT, UNIT, &bars[k]);
      }
    }
  }
  __syncwarp();
  if (PDL) grid_dependency_wait();
  stage_activation(args.act, nb, smem, args.status);
  if (PDL) grid_dependents_launch();

  const int8_t *values = reinterpret_cast<const int8_t *>(smem + MatvecSmem::act_values(nb));
  const float *ascale = reinterpret_cast<const float *>(smem + MatvecSmem::act_scale(nb));
  const int16_t *asums = reinterpret_cast<const int16_t *>(smem + MatvecSmem::act_sums(nb));
  const int *aasum = reinterpret_cast<const int *>(smem + MatvecSmem::act_asum(nb));

  int i = 0;
  for (long u = u0 + warp; u < u1; u += kWarps, ++i) {
    const int k = i % kDepth;
    const unsigned parity = (unsigned)(i / kDepth) & 1u;
    if (!mbar_wait_bounded(&bars[k], parity, args.status)) break;
    const uint8_t *slot = slots + k * UNIT;
    const int t = (int)(u / nb), b = (int)(u % nb);
    const int row = t * kTileRows + lane;
    int dot = 0, dot2 = 0;
    float term;
    if (KIND == 35) {
      tq2_unit(slot, values + b * 256, aasum[b], ascale[b], lane, dot, term);
    } else {
      q2k_unit(slot, values + b * 256, asums + b * 16, ascale[b], lane, dot, dot2, term);
    }
    __syncwarp();
    // refill this slot with the warp's unit kDepth iterations ahead
    const long un = u + (long)kDepth * kWarps;
    if (lane == 0 && un < u1) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars[k], UNIT);
      bulk_g2s(slots + k * UNIT, args.w + un * UNIT, UNIT, &bars[k]);
    }
    if (MODE == kModeInts) {
      if (row < args.rows) {
        args.ints[(size_t)row * nb + b] = dot;
        if (KIND == 10) args.ints2[(size_t)row * nb + b] = dot2;
      }
      continue;
    }
    // publish this unit's terms; the warp that completes the tile sums them
    float *prow = args.partial + ((size_t)t * nb + b) * kTileRows;
    prow[lane] = term;
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(&args.tile_cnt[t], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev == (unsigned)(nb - 1)) {
      __threadfence();
      const float *pt = args.partial + (size_t)t * nb * kTileRows;
      float sum = 0.0f;
      for (int bb = 0; bb < nb; ++bb) sum = __fadd_rn(sum, __ldcg(pt + bb * kTileRows + lane));
      if (row < args.rows) {
        if (!is_finite_f(sum)) report(args.status, kStatusNonfinite);
        args.y[row] = sum;
      }
      if (lane == 0) args.tile_cnt[t] = 0u;
    }
  }
  // never leave bulk copies in flight into shared memory at exit: drain
  // any slot that was armed but not consumed (only after a timeout break)
  for (long u = u0 + warp + (long)i * kWarps; u < u1 && u < u0 + warp + (long)(i + kDepth) * kWarps;
       u += kWarps, ++i) {
    const int k = i % kDepth;
    mbar_wait_bounded(&bars[k], (unsigned)(i / kDepth) & 1u, args.status);
  }
}

// ---- upload-time repack: reference row-major blocks -> tiled units ---------
// One thread per (unit, lane).  src is the reference byte layout.
template <int KIND>
__global__ void repack_kernel(const uint8_t *__restrict__ src, int rows, int nb, int ntiles,
                              uint8_t *__restrict__ dst) {
  constexpr int UNIT = UnitTraits<KIND>::bytes;
  constexpr int BB = KIND == 35 ? 66 : 84;
  long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long total = (long)ntiles * nb * kTileRows;
  if (gid >= total) return;
  int lane = (int)(gid % kTileRows);
  long u = gid / kTileRows;
  int t = (int)(u / nb), b = (int)(u % nb);
  int row = t * kTileRows + lane;
  uint8_t *unit = dst + u * UNIT;
  uint8_t blk[BB];
  if (row < rows) {
    const uint8_t *s = src + ((size_t)row * nb + b) * BB;
    for (int i = 0; i < BB; ++i) blk[i] = s[i];
  } else {
    for (int i = 0; i < BB; ++i) blk[i] = 0;
  }
  const int qoff = KIND == 35 ? 0 : 16;
  for (int c = 0; c < 4; ++c)
    for (int i = 0; i < 16; ++i) unit[(c * 32 + lane) * 16 + i] = blk[qoff + c * 16 + i];
  if (KIND == 35) {
    unit[2048 + lane * 2] = blk[64];
    unit[2048 + lane * 2 + 1] = blk[65];
  } else {
    for (int i = 0; i < 16; ++i) unit[2048 + lane * 16 + i] = blk[i];
    unit[2560 + lane * 2] = blk[80];
    unit[2560 + lane * 2 + 1] = blk[81];
    unit[2624 + lane * 2] = blk[82];
    unit[2624 + lane * 2 + 1] = blk[83];
  }
}

}  // namespace prism
