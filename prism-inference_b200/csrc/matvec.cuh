// matvec.cuh -- batch-1 packed ternary / 2-bit projections on sm_100a.
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
// One launch serves a GROUP of up to four sibling weights that share their
// input (the reference's project_group_into, src/graph.rs:1869), e.g.
// attn_qkv + attn_gate + ssm_beta + ssm_alpha.  Persistent CTAs loop over
// the concatenated tiles (t = blockIdx.x, += gridDim.x).  A tile is streamed
// into shared memory by 1-D bulk async copies (cp.async.bulk, one mbarrier
// per unit) two tiles ahead (double buffer).  Warp w (of 16) computes units
// b = w, w+16, ...: the 32 lanes cover the H rows x 4 chunks (L = 32/H lanes
// per row), weights are lane-private 16-byte shared loads, activations are
// broadcast 16-byte shared loads, byte products use dp4a and per-row integer
// partials combine exactly with shuffles.  Terms go to shared memory; then
// H threads run each row's chain in block order.
//
// Prologues build the Q8_K activation in shared memory, every CTA the same
// bytes: from AoS Q8_K blocks, from f32, from RMSNorm(f32) (the reference's
// normalize-then-prepare, src/kernels.rs:3388-3418 + 463-522), or from
// SwiGLU(up, gate) (src/graph.rs:121-131).  Epilogues store y, add a
// residual (src/kernels.rs:2896-2919), or reduce the greedy argmax
// (src/runtime.rs:2630-2678) with the logits.
#pragma once

#include "common.cuh"
#include "q8k.cuh"

namespace prism {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxNb = 64;     // columns <= 16384 per projection
constexpr int kMaxGroup = 4;   // sibling weights per launch
constexpr int kMaxPrefetch = 8;  // L2 prefetch ranges per launch

__host__ __device__ constexpr int unit_bytes(int kind, int h) {
  return (kind == 35 ? 66 : 84) * h;
}

// Shared-memory layout (dynamic smem), all offsets 16-byte aligned.  `h` is
// the largest tile height in the group (tile buffers are sized for it);
// `upt` is the units per tile (nb, or 2*nb for the up+gate pair); `nbuf`
// tile buffers; `stage_n` floats of staged f32 inputs (x, then the RMSNorm
// weight), 0 when the prologue reads them in place.
struct MatvecSmem {
  int nb, h, unit, upt, nbuf, stage_n;
  __host__ __device__ MatvecSmem(int nb_, int h_, int unit_, int upt_, int nbuf_ = 2,
                                 int stage_n_ = 0)
      : nb(nb_), h(h_), unit(unit_), upt(upt_), nbuf(nbuf_), stage_n(stage_n_) {}
  __host__ __device__ int act_values() const { return 0; }
  __host__ __device__ int act_scale() const { return nb * 256; }
  __host__ __device__ int act_sums() const { return act_scale() + nb * 4; }
  __host__ __device__ int act_asum() const { return act_sums() + nb * 32; }
  __host__ __device__ int red() const { return (act_asum() + nb * 4 + 15) / 16 * 16; }
  __host__ __device__ int terms() const { return red() + kWarps * 16; }
  // terms are double-buffered: one tile's chains run while the next tile's
  // dots fill the other buffer
  __host__ __device__ int bars() const { return (terms() + 2 * upt * h * 4 + 15) / 16 * 16; }
  __host__ __device__ int stage() const { return (bars() + nbuf * upt * 8 + 15) / 16 * 16; }
  __host__ __device__ int bufs() const { return (stage() + stage_n * 4 + 127) / 128 * 128; }
  __host__ __device__ int tile_bytes() const { return upt * unit; }
  __host__ __device__ int total() const { return bufs() + nbuf * tile_bytes(); }
};

// kProGated: x = RMSNorm(o_h) * w * SiLU(z_h) per head of head_dim values
// (the Gated DeltaNet output, reference src/kernels.rs:3589-3625 Source),
// in0 = o, zgate = SiLU(z) (already applied), norm_w = w [head_dim].
enum Prologue : int { kProQ8K = 0, kProF32 = 1, kProRmsNorm = 2, kProGated = 3 };
// kEpiSwiglu: w[0] = ffn_up, w[1] = ffn_gate (same geometry); each tile of
// rows is projected through both and y = up * silu(gate) is stored in
// w[0].y (reference src/graph.rs:121-131 SwiGLU).
enum Epilogue : int { kEpiStore = 0, kEpiArgmax = 1, kEpiInts = 2, kEpiSwiglu = 3 };

struct MvWeight {
  const uint8_t *units = nullptr;
  int h = 32, ntiles = 0, rows = 0;
  float *y = nullptr;               // output rows (kEpiStore / kEpiArgmax logits)
  const float *residual = nullptr;  // y[r] = residual[r] + chain (may alias y)
  int32_t *ints = nullptr;          // kEpiInts: rows*nb block dots
  int32_t *ints2 = nullptr;         // kEpiInts, Q2_K min sums
};

struct MvArgs {
  MvWeight w[kMaxGroup];
  int count = 1;
  int nb = 0;
  int tile_start[kMaxGroup + 1] = {0, 0, 0, 0, 0};
  int prologue = kProQ8K;
  const void *in0 = nullptr;        // Q8_K AoS | f32 x | f32 x
  const float *norm_w = nullptr;    // kProRmsNorm weight
  const float *zgate = nullptr;     // kProGated: [heads * head_dim]
  int gheads = 0, ghd = 0;          // kProGated geometry
  float eps = 0.0f;
  int pinned = 0;                   // pinned Q8_K rounding
  unsigned long long *argmax_key = nullptr;
  unsigned *status = nullptr;
  int nbuf = 2;                     // tile buffers (tiles in flight per CTA)
  int stage = 0;                    // 1: stage f32 inputs in shared memory first
  // L2 prefetch of later kernels' operands (weights, recurrent state): the
  // grid splits each range; 16-byte aligned, sizes multiples of 16
  const uint8_t *pf[kMaxPrefetch] = {};
  unsigned pf_bytes[kMaxPrefetch] = {};
  // optional timeline (globaltimer ns): CTA 0's [0] entry, [1] past the grid
  // dependency, [2] input staged, [3] first tile resident, [4] its dots,
  // [5] its chains, [6] exit; [7] the last CTA's exit
  unsigned long long *trace = nullptr;
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

// One unit of one weight: this lane's row gets its block's term and the
// exact integer dots (dot, dot2 = Q2_K min sum).
template <int KIND, int H>
__device__ __forceinline__ void unit_terms(const uint8_t *unit, const int8_t *av, int asum,
                                           const int16_t *gs, float s, int lane, int &dot,
                                           int &dot2, float &term) {
  const int r = lane % H;
  if (KIND == 35) {
    dot = row_allreduce<H>(tq2_lane_partial<H>(unit, av, lane)) - asum;
    dot2 = 0;
    const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(unit + 64 * H)[r]);
    term = __fmul_rn((float)dot, __fmul_rn(d, s));
  } else {
    const uint4 sc = reinterpret_cast<const uint4 *>(unit + 64 * H)[r];
    dot = row_allreduce<H>(q2k_lane_partial<H>(unit, av, sc, lane));
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
}

// ---- prologues ----------------------------------------------------------

// Store one quantized block (lane holds q[8] of values 8l..8l+7) into the
// structure-of-arrays activation layout in shared memory.
__device__ __forceinline__ void store_q8k_soa(const MatvecSmem &L, uint8_t *smem, int b,
                                              int lane, float scale, const int8_t (&q)[8],
                                              int pair_sum) {
  int8_t *values = reinterpret_cast<int8_t *>(smem + L.act_values()) + b * 256;
  uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) |
                ((uint32_t)(uint8_t)q[2] << 16) | ((uint32_t)(uint8_t)q[3] << 24);
  uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) |
                ((uint32_t)(uint8_t)q[6] << 16) | ((uint32_t)(uint8_t)q[7] << 24);
  reinterpret_cast<uint2 *>(values)[lane] = make_uint2(w0, w1);
  if ((lane & 1) == 0)
    reinterpret_cast<int16_t *>(smem + L.act_sums())[b * 16 + (lane >> 1)] = (int16_t)pair_sum;
  int tot = pair_sum;
#pragma unroll
  for (int off = 2; off < 32; off <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (lane == 0) {
    reinterpret_cast<float *>(smem + L.act_scale())[b] = scale;
    reinterpret_cast<int *>(smem + L.act_asum())[b] = tot;
  }
}

// Stage AoS Q8_K blocks (4-byte aligned) into the SoA layout.
__device__ __forceinline__ void stage_q8k_aos(const uint8_t *act, const MatvecSmem &L,
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
}

// Sum of squares of x[0..n) in binary64 (reference rms_norm_scale_inner,
// src/kernels.rs:3823-3878), block-wide, deterministic order.
__device__ __forceinline__ double block_sumsq_f64(const float *x, int n, double *red) {
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    s += (double)__fmul_rn(v, v);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  __syncthreads();
  return t;
}

// Build the Q8_K activation in shared memory from an f32 vector:
//   kProF32:     x
//   kProRmsNorm: (x * scale) * w, scale = 1/sqrt(mean(x^2) + eps)
__device__ __forceinline__ void stage_from_f32(const MvArgs &a, const MatvecSmem &L,
                                               uint8_t *smem, const float *x_override = nullptr,
                                               const float *w_override = nullptr) {
  const int nb = L.nb, n = nb * 256;
  const float *x = x_override ? x_override : static_cast<const float *>(a.in0);
  const float *norm_w = w_override ? w_override : a.norm_w;
  float scale = 1.0f;
  if (a.prologue == kProRmsNorm) {
    double *red = reinterpret_cast<double *>(smem + L.red());
    const double sum = block_sumsq_f64(x, n, red);
    const float mean = (float)(sum / (double)n);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
    if (!is_finite_f(scale) || !(scale > 0.0f)) {
      if (threadIdx.x == 0) report(a.status, kStatusNonfinite);
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < nb; b += blockDim.x >> 5) {
    const int base = b * 256 + lane * 8;
    float v[8];
    const float4 x0 = *reinterpret_cast<const float4 *>(x + base);
    const float4 x1 = *reinterpret_cast<const float4 *>(x + base + 4);
    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
    v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
    if (a.prologue == kProRmsNorm) {
      const float4 w0 = *reinterpret_cast<const float4 *>(norm_w + base);
      const float4 w1 = *reinterpret_cast<const float4 *>(norm_w + base + 4);
      const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], scale), w[i]);
    }
    float qscale;
    int8_t q[8];
    int pair_sum;
    unsigned st = q8k_quantize_regs(v, lane, a.pinned != 0, qscale, q, pair_sum);
    if (st && lane == 0) report(a.status, st);
    store_q8k_soa(L, smem, b, lane, qscale, q, pair_sum);
  }
}

// This CTA's share of the launch's L2 prefetch ranges (one thread), in
// pieces of at most 32 KB.
__device__ __forceinline__ void prefetch_l2_share(const MvArgs &a) {
  for (int r = 0; r < kMaxPrefetch; ++r) {
    const unsigned bytes = a.pf_bytes[r];
    if (!bytes) continue;
    const unsigned chunk = (bytes / gridDim.x + 15u) / 16u * 16u;
    const unsigned lo = blockIdx.x * chunk;
    const unsigned hi = min(bytes, lo + chunk);
    for (unsigned o = lo; o < hi; o += 32768u) {
      const unsigned len = min(32768u, hi - o);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.pf[r] + o), "r"(len)
                   : "memory");
    }
  }
}

// Gated output norm of `heads` heads of S (== 128) values, one warp per
// head: y = RMSNorm(o_h) * w * g_h with g = SiLU(z) given, the binary64 sum
// of squares in the order of a 512-thread block sum over the head
// (gdn_decode_kernel's tail).  y may alias o.
__device__ __forceinline__ void gated_heads_norm(int heads, int S, float eps, const float *o_all,
                                                 const float *g_all, const float *w, float *out,
                                                 float *copy_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int h = warp; h < heads; h += (int)(blockDim.x >> 5)) {
    const float *o = o_all + h * S;
    double t = 0.0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float v = o[32 * q + lane];
      double sq = (double)__fmul_rn(v, v);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
      t += sq;
    }
    const float mean = (float)(t / (double)S);
    const float nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = 32 * q + lane;
      const float normed = __fmul_rn(__fmul_rn(o[i], nscale), w[i]);
      const float y = __fmul_rn(normed, g_all[h * S + i]);
      out[h * S + i] = y;
      if (copy_out) copy_out[h * S + i] = y;
    }
  }
}

// Copy n floats (n % 4 == 0, 16-byte aligned) into shared memory, all
// threads, every load in flight before the stores.
__device__ __forceinline__ void load_f32_to_smem(float *dst, const float *src, int n) {
#pragma unroll 4
  for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4)
    *reinterpret_cast<float4 *>(dst + i) = *reinterpret_cast<const float4 *>(src + i);
}

// Issue the bulk copies of one tile into buffer `buf` (one mbarrier per unit).
__device__ __forceinline__ void issue_tile(const uint8_t *src, int nb, int unit, uint8_t *buf,
                                           uint64_t *bars) {
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    mbar_arrive_expect_tx(&bars[b], unit);
    bulk_g2s(buf + b * unit, src + (long)b * unit, unit, &bars[b]);
  }
}

__device__ __forceinline__ int group_of(const MvArgs &a, int t) {
  int g = 0;
#pragma unroll
  for (int i = 1; i < kMaxGroup; ++i)
    if (i < a.count && t >= a.tile_start[i]) g = i;
  return g;
}

template <int EPI>
__device__ __forceinline__ void issue_group_tile(const MvArgs &a, int kind, int t, uint8_t *buf,
                                                 uint64_t *bars) {
  if (EPI == kEpiSwiglu) {
    // units [0, nb) from ffn_up tile t, [nb, 2nb) from ffn_gate tile t
    const int unit = unit_bytes(kind, a.w[0].h);
    issue_tile(a.w[0].units + (long)t * a.nb * unit, a.nb, unit, buf, bars);
    issue_tile(a.w[1].units + (long)t * a.nb * unit, a.nb, unit, buf + a.nb * unit,
               bars + a.nb);
    return;
  }
  const int g = group_of(a, t);
  const MvWeight &w = a.w[g];
  const int unit = unit_bytes(kind, w.h);
  const int lt = t - a.tile_start[g];
  issue_tile(w.units + (long)lt * a.nb * unit, a.nb, unit, buf, bars);
}

// Sortable key of a finite float (larger value -> larger key), with the
// lowest index winning ties: the reference's greedy selection order.
__device__ __forceinline__ unsigned long long argmax_key(float v, int index) {
  unsigned u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (unsigned)index);
}

template <int KIND, int EPI>
__global__ void __launch_bounds__(kThreads) matvec_kernel(MvArgs args) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nb = args.nb;
  constexpr bool PAIR = EPI == kEpiSwiglu;
  const int upt = PAIR ? 2 * nb : nb;
  int hmax = 8;
  for (int g = 0; g < args.count; ++g) hmax = max(hmax, args.w[g].h);
  const int nbuf = args.nbuf, n = nb * 256;
  const bool gated = args.prologue == kProGated;
  const bool staged = gated || (args.stage && args.prologue != kProQ8K);
  const MatvecSmem L(nb, hmax, unit_bytes(KIND, hmax), upt, nbuf,
                     !staged                          ? 0
                     : gated                          ? 2 * n + args.ghd
                     : args.prologue == kProRmsNorm   ? 2 * n
                                                      : n);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars());  // [nbuf][upt]
  uint8_t *bufs = smem + L.bufs();                                  // [nbuf][tile]
  float *terms2 = reinterpret_cast<float *>(smem + L.terms());      // [2][upt][H]
  float *xs = reinterpret_cast<float *>(smem + L.stage());          // [n] x, [n] norm weight
  const int ntiles = PAIR ? args.w[0].ntiles : args.tile_start[args.count];
  trace_stamp(args.trace, 0);

  for (int i = threadIdx.x; i < nbuf * upt; i += blockDim.x) {
    mbar_init(&bars[i], 1);
    mbar_init_fence();
  }
  __syncthreads();
  // Weights never depend on the previous kernel: stream this CTA's first
  // nbuf tiles, and stage the RMSNorm weight, before waiting on the grid
  // dependency.
  const int t0 = blockIdx.x;
  if (threadIdx.x == 32) prefetch_l2_share(args);
  for (int j = 0; j < nbuf; ++j) {
    const int tj = t0 + j * (int)gridDim.x;
    if (tj < ntiles) issue_group_tile<EPI>(args, KIND, tj, bufs + j * L.tile_bytes(), bars + j * upt);
  }
  if (staged && args.prologue == kProRmsNorm) load_f32_to_smem(xs + n, args.norm_w, n);
  if (gated) load_f32_to_smem(xs + 2 * n, args.norm_w, args.ghd);
  grid_dependency_wait();
  trace_stamp(args.trace, 1);
  if (args.prologue == kProQ8K) {
    stage_q8k_aos(static_cast<const uint8_t *>(args.in0), L, smem, args.status);
  } else if (gated) {
    // o and z in one round of loads, the gated norm in place over o, then
    // the quantization of the gated vector
    load_f32_to_smem(xs, static_cast<const float *>(args.in0), n);
    load_f32_to_smem(xs + n, args.zgate, n);
    __syncthreads();
    gated_heads_norm(args.gheads, args.ghd, args.eps, xs, xs + n, xs + 2 * n, xs, nullptr);
    __syncthreads();
    stage_from_f32(args, L, smem, xs, nullptr);
  } else if (staged) {
    // the input arrives with one round of loads, then the prologue works
    // from shared memory
    load_f32_to_smem(xs, static_cast<const float *>(args.in0), n);
    __syncthreads();
    stage_from_f32(args, L, smem, xs, xs + n);
  } else {
    stage_from_f32(args, L, smem);
  }
  __syncthreads();
  trace_stamp(args.trace, 2);
  grid_dependents_launch();

  const int8_t *values = reinterpret_cast<const int8_t *>(smem + L.act_values());
  const float *ascale = reinterpret_cast<const float *>(smem + L.act_scale());
  const int16_t *asums = reinterpret_cast<const int16_t *>(smem + L.act_sums());
  const int *aasum = reinterpret_cast<const int *>(smem + L.act_asum());
  unsigned long long best = 0ull;

  bool ok = true;
  int it = 0;
  for (int t = t0; t < ntiles; t += gridDim.x, ++it) {
    const int k = it % nbuf;
    const unsigned parity = (unsigned)(it / nbuf) & 1u;
    uint8_t *buf = bufs + k * L.tile_bytes();
    uint64_t *bk = bars + k * upt;
    const int g = PAIR ? 0 : group_of(args, t);
    const MvWeight &w = args.w[g];
    const int H = w.h;
    const int unit = unit_bytes(KIND, H);
    const int lt = t - (PAIR ? 0 : args.tile_start[g]);
    const int r = lane % H;
    const int row = lt * H + r;
    float *terms = terms2 + (it & 1) * upt * hmax;
    for (int u = warp; u < upt; u += kWarps) {
      if (!mbar_wait_bounded(&bk[u], parity, args.status)) {
        ok = false;
        break;
      }
      if (it == 0 && u == warp) trace_stamp(args.trace, 3);
      const int b = PAIR && u >= nb ? u - nb : u;  // activation block
      const uint8_t *up = buf + u * unit;
      const int8_t *av = values + b * 256;
      int dot, dot2;
      float term;
      if (H == 32)
        unit_terms<KIND, 32>(up, av, aasum[b], asums + b * 16, ascale[b], lane, dot, dot2, term);
      else if (H == 16)
        unit_terms<KIND, 16>(up, av, aasum[b], asums + b * 16, ascale[b], lane, dot, dot2, term);
      else
        unit_terms<KIND, 8>(up, av, aasum[b], asums + b * 16, ascale[b], lane, dot, dot2, term);
      if (lane < H) {
        if (EPI == kEpiInts) {
          if (row < w.rows) {
            w.ints[(size_t)row * nb + b] = dot;
            if (KIND == 10) w.ints2[(size_t)row * nb + b] = dot2;
          }
        } else {
          terms[u * H + r] = term;
        }
      }
    }
    // the tile's terms are complete and its data consumed: refill the
    // buffer with the tile nbuf steps ahead, then run the chains (threads
    // below H) while the other warps go on to the next tile's dots
    if (!__syncthreads_and(ok)) break;
    if (it == 0) trace_stamp(args.trace, 4);
    const int tn = t + nbuf * (int)gridDim.x;
    if (tn < ntiles) {
      fence_proxy_async_smem();
      issue_group_tile<EPI>(args, KIND, tn, buf, bk);
    }
    if (EPI != kEpiInts && threadIdx.x < H) {
      // the reference's chain: sum = 0; sum += term_b for b in order
      float sum = 0.0f;
      for (int b = 0; b < nb; ++b) sum = __fadd_rn(sum, terms[b * H + threadIdx.x]);
      const int orow = lt * H + threadIdx.x;
      if (PAIR) {
        float gsum = 0.0f;
        for (int b = nb; b < 2 * nb; ++b) gsum = __fadd_rn(gsum, terms[b * H + threadIdx.x]);
        if (orow < w.rows) {
          const float h = __fmul_rn(sum, silu_f(gsum));
          if (!is_finite_f(sum) || !is_finite_f(gsum)) report(args.status, kStatusNonfinite);
          w.y[orow] = h;
        }
      } else if (orow < w.rows) {
        if (w.residual) sum = __fadd_rn(w.residual[orow], sum);
        if (!is_finite_f(sum)) report(args.status, kStatusNonfinite);
        if (w.y) w.y[orow] = sum;
        if (EPI == kEpiArgmax) {
          const unsigned long long key = argmax_key(sum, orow);
          best = key > best ? key : best;
        }
      }
    }
    if (it == 0) trace_stamp(args.trace, 5);
  }
  if (EPI == kEpiArgmax) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0 && best) atomicMax(args.argmax_key, best);
  }
  if (!ok) {
    // a wait expired: drain every armed copy (bounded) before exiting
    for (int j = 0; j < nbuf; ++j) {
      const int tj = t0 + (it + j) * (int)gridDim.x;
      if (tj >= ntiles) break;
      const int kj = (it + j) % nbuf;
      for (int u = threadIdx.x; u < upt; u += blockDim.x)
        mbar_wait_bounded(&bars[kj * upt + u], (unsigned)((it + j) / nbuf) & 1u, args.status);
    }
  }
  trace_exit(args.trace);
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
