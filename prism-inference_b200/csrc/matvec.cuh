// matvec.cuh -- batch-1 packed ternary / 2-bit projection on sm_100a.
//
// y[r] = sum_b term(r, b): term is the reference's per-block binary32
// contribution and the sum is the reference's sequential binary32 chain over
// blocks (TQ2_0: reference src/kernels/tquants.rs:270-287; Q2_K:
// src/kernels/kquants.rs:346-420 kind 10).  Integer block dots are exact, so
// outputs are bit-identical to the reference's CPU kernels.
//
// Device weight layout ("tiled", built once at upload).  Rows are grouped in
// tiles of H rows (H = 32, 16 or 8, chosen per weight so that small matrices
// still yield enough tiles for every SM); the last tile is zero padded.  A
// UNIT is one tile x one 256-column block; a tile's nb units are contiguous:
//   TQ2_0 unit (66 H B): qs[4 chunks][H rows][16 B] | d[H] fp16
//   Q2_K  unit (84 H B): qs[4][H][16 B] | scales[H][16 B] | d[H] | dmin[H]
// Chunk c of a row's block is bytes 16c..16c+15 of its 64 quant bytes.  The
// layout holds exactly the packed bytes (plus tile padding), so HBM traffic
// equals the reference's packed size.
//
// Execution: persistent CTAs loop over tiles (t = blockIdx.x, += gridDim.x).
// A tile is streamed into shared memory by 1-D bulk async copies
// (cp.async.bulk, one mbarrier per unit) two tiles ahead (double buffer), so
// the next tile's bytes are in flight while the current one is computed.
// Warp w computes units b = w, w+8, ...: the 32 lanes cover the H rows x 4
// chunks (L = 32/H lanes per row), weights are lane-private 16-byte shared
// loads, activations are broadcast 16-byte shared loads, byte products use
// dp4a and per-row integer partials combine exactly with shuffles.  Terms go
// to shared memory; then H threads run each row's chain in block order.
#pragma once

#include "common.cuh"
#include "q8k.cuh"

namespace prism {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxNb = 64;  // columns <= 16384 per projection

__host__ __device__ constexpr int unit_bytes(int kind, int h) {
  return (kind == 35 ? 66 : 84) * h;
}

// Shared-memory layout (dynamic smem), all offsets 16-byte aligned.
struct MatvecSmem {
  int nb, h, unit;
  __host__ __device__ MatvecSmem(int nb_, int h_, int unit_) : nb(nb_), h(h_), unit(unit_) {}
  __host__ __device__ int act_values() const { return 0; }
  __host__ __device__ int act_scale() const { return nb * 256; }
  __host__ __device__ int act_sums() const { return act_scale() + nb * 4; }
  __host__ __device__ int act_asum() const { return act_sums() + nb * 32; }
  __host__ __device__ int terms() const { return (act_asum() + nb * 4 + 15) / 16 * 16; }
  __host__ __device__ int bars() const { return (terms() + nb * h * 4 + 15) / 16 * 16; }
  __host__ __device__ int bufs() const { return (bars() + 2 * nb * 8 + 127) / 128 * 128; }
  __host__ __device__ int tile_bytes() const { return nb * unit; }
  __host__ __device__ int total() const { return bufs() + 2 * tile_bytes(); }
};

enum MatvecMode : int {
  kModeOutput = 0,  // y = W x
  kModeInts = 1,    // exact per-block integer dots to ints / ints2
};

struct MatvecArgs {
  const uint8_t *w;      // tiled units
  const uint8_t *act;    // nb AoS Q8_K blocks (4-byte aligned)
  int nb;                // blocks per row
  int ntiles;            // H-row tiles
  int rows;              // true rows
  float *y;              // rows floats (kModeOutput)
  int32_t *ints;         // rows*nb (kModeInts)
  int32_t *ints2;        // rows*nb (kModeInts, Q2_K min sums)
  unsigned *status;
};

__device__ __forceinline__ unsigned byte_of(const uint4 &v, int g) {
  unsigned w = (g < 4) ? v.x : (g < 8) ? v.y : (g < 12) ? v.z : v.w;
  return (w >> (8 * (g & 3))) & 0xffu;
}

// Lane partial of a TQ2_0 unit: sum over this lane's chunks of code*q,
// with plane j scaled by 4^j folded back exactly.
template <int H>
__device__ __forceinline__ int tq2_lane_partial(const uint8_t *unit, const int8_t *av,
                                                int lane) {
  constexpr int L = 32 / H;
  const int r = lane % H, s = lane / H;
  const uint4 *qs = reinterpret_cast<const uint4 *>(unit);
  int acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;
#pragma unroll
  for (int i = 0; i < 4 / L; ++i) {
    const int c = s + i * L;
    uint4 wq = qs[c * H + r];
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
  return acc0 + (acc1 >> 2) + (acc2 >> 4) + (acc3 >> 6);
}

// Lane partial of a Q2_K unit's scaled integer sum: sum_g sc_g * sum q*a
// over this lane's chunks (each chunk x plane is exactly one 16-group).
template <int H>
__device__ __forceinline__ int q2k_lane_partial(const uint8_t *unit, const int8_t *av,
                                                const uint4 &sc, int lane) {
  constexpr int L = 32 / H;
  const int r = lane % H, s = lane / H;
  const uint4 *qs = reinterpret_cast<const uint4 *>(unit);
  int is = 0;
#pragma unroll
  for (int i = 0; i < 4 / L; ++i) {
    const int c = s + i * L;
    uint4 wq = qs[c * H + r];
    const int8_t *base = av + (c >> 1) * 128 + (c & 1) * 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const unsigned m = 0x03030303u << (2 * j);
      int4 a = *reinterpret_cast<const int4 *>(base + 32 * j);
      int acc = dp4a_us(wq.x & m, a.x, 0);
      acc = dp4a_us(wq.y & m, a.y, acc);
      acc = dp4a_us(wq.z & m, a.z, acc);
      acc = dp4a_us(wq.w & m, a.w, acc);
      // group g = 8*(c/2) + 2*j + (c%2); c is lane dependent when L > 1
      const int g = 8 * (c >> 1) + 2 * j + (c & 1);
      is += (int)(byte_of(sc, g) & 15u) * (acc >> (2 * j));
    }
  }
  return is;
}

// Sum a per-lane integer over the L lanes that share a row (exact).
template <int H>
__device__ __forceinline__ int row_allreduce(int v) {
#pragma unroll
  for (int off = H; off < 32; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Stage the Q8_K activation (AoS, 4-byte aligned) into shared memory as
// values[nb][256] | scale[nb] | sums[nb][16] | asum[nb].
__device__ __forceinline__ void stage_activation(const uint8_t *act, const MatvecSmem &L,
                                                 uint8_t *smem, unsigned *status) {
  const int nb = L.nb;
  int8_t *values = reinterpret_cast<int8_t *>(smem + L.act_values());
  float *scale = reinterpret_cast<float *>(smem + L.act_scale());
  int16_t *sums = reinterpret_cast<int16_t *>(smem + L.act_sums());
  int *asum = reinterpret_cast<int *>(smem + L.act_asum());
  const uint32_t *src = reinterpret_cast<const uint32_t *>(act);
  // 73 words per block: word 0 scale, words 1..64 values, 65..72 sums
  for (int i = threadIdx.x; i < nb * 73; i += blockDim.x) {
    int b = i / 73, k = i - b * 73;
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

// Issue the bulk copies of tile t into buffer `buf` (one mbarrier per unit).
__device__ __forceinline__ void issue_tile(const uint8_t *w, long t, int nb, int unit,
                                           uint8_t *buf, uint64_t *bars) {
  const uint8_t *src = w + t * (long)nb * unit;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    mbar_arrive_expect_tx(&bars[b], unit);
    bulk_g2s(buf + b * unit, src + (long)b * unit, unit, &bars[b]);
  }
}

template <int KIND, int H, int MODE, bool PDL>
__global__ void __launch_bounds__(kThreads) matvec_kernel(MatvecArgs args) {
  constexpr int UNIT = unit_bytes(KIND, H);
  extern __shared__ __align__(128) uint8_t smem[];
  const int nb = args.nb;
  const MatvecSmem L(nb, H, UNIT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars());  // [2][nb]
  uint8_t *bufs = smem + L.bufs();                                  // [2][tile]
  float *terms = reinterpret_cast<float *>(smem + L.terms());       // [nb][H]

  for (int i = threadIdx.x; i < 2 * nb; i += blockDim.x) {
    mbar_init(&bars[i], 1);
    mbar_init_fence();
  }
  __syncthreads();
  // Weights never depend on the previous kernel: stream the first two tiles
  // before waiting on the grid dependency.
  const int t0 = blockIdx.x;
  if (t0 < args.ntiles) issue_tile(args.w, t0, nb, UNIT, bufs, bars);
  if (t0 + (int)gridDim.x < args.ntiles)
    issue_tile(args.w, t0 + gridDim.x, nb, UNIT, bufs + L.tile_bytes(), bars + nb);
  if (PDL) grid_dependency_wait();
  stage_activation(args.act, L, smem, args.status);
  if (PDL) grid_dependents_launch();

  const int8_t *values = reinterpret_cast<const int8_t *>(smem + L.act_values());
  const float *ascale = reinterpret_cast<const float *>(smem + L.act_scale());
  const int16_t *asums = reinterpret_cast<const int16_t *>(smem + L.act_sums());
  const int *aasum = reinterpret_cast<const int *>(smem + L.act_asum());
  const int r = lane % H;

  bool ok = true;
  int it = 0;
  for (int t = t0; t < args.ntiles; t += gridDim.x, ++it) {
    const int k = it & 1;
    const unsigned parity = (unsigned)(it >> 1) & 1u;
    uint8_t *buf = bufs + k * L.tile_bytes();
    uint64_t *bk = bars + k * nb;
    const int row = t * H + r;
    for (int b = warp; b < nb; b += kWarps) {
      if (!mbar_wait_bounded(&bk[b], parity, args.status)) {
        ok = false;
        break;
      }
      const uint8_t *unit = buf + b * UNIT;
      const int8_t *av = values + b * 256;
      const float s = ascale[b];
      int dot, dot2 = 0;
      float term;
      if (KIND == 35) {
        dot = row_allreduce<H>(tq2_lane_partial<H>(unit, av, lane)) - aasum[b];
        const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(unit + 64 * H)[r]);
        term = __fmul_rn((float)dot, __fmul_rn(d, s));
      } else {
        const uint4 sc = reinterpret_cast<const uint4 *>(unit + 64 * H)[r];
        dot = row_allreduce<H>(q2k_lane_partial<H>(unit, av, sc, lane));
        const int16_t *gs = asums + b * 16;
        int ms = 0;
#pragma unroll
        for (int g = 0; g < 16; ++g) ms += (int)gs[g] * (int)(byte_of(sc, g) >> 4);
        dot2 = ms;
        const uint16_t *dd = reinterpret_cast<const uint16_t *>(unit + 80 * H);
        const float d = half_bits_to_float(dd[r]);
        const float dmin = half_bits_to_float(dd[H + r]);
        const float t1 = __fmul_rn(__fmul_rn(s, d), (float)dot);
        const float t2 = __fmul_rn(__fmul_rn(s, dmin), (float)ms);
        term = __fsub_rn(t1, t2);
      }
      if (lane < H) {
        if (MODE == kModeInts) {
          if (row < args.rows) {
            args.ints[(size_t)row * nb + b] = dot;
            if (KIND == 10) args.ints2[(size_t)row * nb + b] = dot2;
          }
        } else {
          terms[b * H + r] = term;
        }
      }
    }
    if (!__syncthreads_and(ok)) break;
    if (MODE == kModeOutput && threadIdx.x < H) {
      // the reference's chain: sum = 0; sum += term_b for b in order
      float sum = 0.0f;
      for (int b = 0; b < nb; ++b) sum = __fadd_rn(sum, terms[b * H + threadIdx.x]);
      const int orow = t * H + threadIdx.x;
      if (orow < args.rows) {
        if (!is_finite_f(sum)) report(args.status, kStatusNonfinite);
        args.y[orow] = sum;
      }
    }
    __syncthreads();
    // refill this buffer with the tile two steps ahead
    const int tn = t + 2 * gridDim.x;
    if (tn < args.ntiles) {
      fence_proxy_async_smem();
      issue_tile(args.w, tn, nb, UNIT, buf, bk);
    }
  }
  if (!ok) {
    // a wait expired: drain every armed copy (bounded) before exiting
    for (int j = 0; j < 2; ++j) {
      const int tj = t0 + (it + j) * gridDim.x;
      if (tj >= args.ntiles) break;
      const int kj = (it + j) & 1;
      for (int b = threadIdx.x; b < nb; b += blockDim.x)
        mbar_wait_bounded(&bars[kj * nb + b], (unsigned)((it + j) >> 1) & 1u, args.status);
    }
  }
}

// ---- upload-time repack: reference row-major blocks -> tiled units ---------
// One thread per (tile, block, row).  src is the reference byte layout.
template <int KIND, int H>
__global__ void repack_kernel(const uint8_t *__restrict__ src, int rows, int nb, int ntiles,
                              uint8_t *__restrict__ dst) {
  constexpr int UNIT = unit_bytes(KIND, H);
  constexpr int BB = KIND == 35 ? 66 : 84;
  long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long total = (long)ntiles * nb * H;
  if (gid >= total) return;
  int r = (int)(gid % H);
  long u = gid / H;
  int t = (int)(u / nb), b = (int)(u % nb);
  int row = t * H + r;
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
    for (int i = 0; i < 16; ++i) unit[(c * H + r) * 16 + i] = blk[qoff + c * 16 + i];
  if (KIND == 35) {
    unit[64 * H + r * 2] = blk[64];
    unit[64 * H + r * 2 + 1] = blk[65];
  } else {
    for (int i = 0; i < 16; ++i) unit[64 * H + r * 16 + i] = blk[i];
    unit[80 * H + r * 2] = blk[80];
    unit[80 * H + r * 2 + 1] = blk[81];
    unit[82 * H + r * 2] = blk[82];
    unit[82 * H + r * 2 + 1] = blk[83];
  }
}

}  // namespace prism
