// kvq.cuh -- the reference's rotated scalar KV codec ("rsq", reference
// src/kv_quant.rs with src/kv_quant/scalar.rs, fitted_scale.rs, tables.rs)
// and the attention over its records (reference src/graph/quantized_kv.rs:
// 1302-1348 attend_head, Source arithmetic) on the device.
//
// Codec (256 channels; every block below has 256 threads, thread i owns
// channel i):
//   - encode: scale = |x|_2 / 16 with |x|^2 a binary64 FMA chain in channel
//     order, rounded to binary32; row = binary32(x / scale) in binary64; three
//     passes of a seeded sign flip then the normalised Walsh-Hadamard
//     transform (butterflies of width 1..128 in binary32, then x 1/16); each
//     coordinate coded as its nearest level (rounded binary32 distances, the
//     first code on ties); version 2 then fits the stored scale to the codes
//     under the reference's rotated-error guard.  The record: binary32 scale,
//     then the codes packed little-endian, 3 or 4 bits each (100 / 132 B).
//   - score: the rotated query against the codes in four binary64 lanes
//     (channel i into lane i % 4, channel order, exact products), reduced
//     ((l0 + l1) + l2) + l3, rounded to binary32, times the record scale.
//   - value scan: binary32 acc_i += (p * scale) * level, positions in order,
//     in the rotated basis; one inverse rotation ends the scan.
// The butterflies of one width are independent, so running them across
// threads keeps every rounding of the sequential transform.  The binary64
// chains whose order is the contract (norm, fitted-scale sums, softmax total)
// run in one thread each; the value scan runs one binary32 chain per channel.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "executor.cuh"
#include "model_kernels.cuh"

namespace prism {

constexpr int kKvqDim = 256;
constexpr int kKvqSplit = 8;        // CTAs (one cluster) per query head
constexpr int kKvqMaxPos = 32768;   // positions one attention launch serves
constexpr int kKvqChunk = 256;      // value-scan staging chunk, positions
constexpr uint64_t kKvqKeySeed = 0x53574946544b5631ull;    // reference KEY_SEED
constexpr uint64_t kKvqValueSeed = 0x5357494654565631ull;  // reference VALUE_SEED

__host__ __device__ constexpr int kvq_record_bytes(int bits) {
  return bits == 3 ? 100 : bits == 4 ? 132 : 0;
}

// The reference's published binary32 Lloyd-Max levels (src/kv_quant/
// tables.rs:10-46), a format table kept bit for bit.
static __constant__ uint32_t kKvqLevel3[8] = {0xc009b97au, 0xbfac0538u, 0xbf418990u,
                                              0xbe7af9f7u, 0x3e7af9f7u, 0x3f418990u,
                                              0x3fac0538u, 0x4009b97au};
static __constant__ uint32_t kKvqLevel4[16] = {
    0xc02ee2bdu, 0xc0046ac7u, 0xbfcf1c25u, 0xbfa0cc2fu, 0xbf713d36u, 0xbf28215bu,
    0xbec6ae44u, 0xbe0379fdu, 0x3e0379fdu, 0x3ec6ae44u, 0x3f28215bu, 0x3f713d36u,
    0x3fa0cc2fu, 0x3fcf1c25u, 0x40046ac7u, 0x402ee2bdu};

// One codec: precision, format version and the three passes' sign bits
// (bit i % 32 of neg[p][i / 32] set: channel i is negated in pass p).
struct KvqCodec {
  int bits;      // 3 or 4
  int version;   // 1, or 2: fitted scale (encoding only)
  uint32_t neg[3][8];
};

// The reference's sign stream (src/kv_quant.rs:409-420, SplitMix64 from the
// seed, bit 0 of each word; passes in order, channels in order).
inline KvqCodec kvq_codec(int bits, uint64_t seed, int version) {
  KvqCodec c{};
  c.bits = bits;
  c.version = version;
  uint64_t s = seed;
  for (int p = 0; p < 3; ++p)
    for (int i = 0; i < kKvqDim; ++i) {
      s += 0x9e3779b97f4a7c15ull;
      uint64_t z = s;
      z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
      z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
      z ^= z >> 31;
      if (z & 1u) c.neg[p][i / 32] |= 1u << (i % 32);
    }
  return c;
}

__device__ __forceinline__ float kvq_level(int bits, int code) {
  return __uint_as_float(bits == 3 ? kKvqLevel3[code & 7] : kKvqLevel4[code & 15]);
}

__device__ __forceinline__ float kvq_sign(const KvqCodec &c, int p, int i, float v) {
  return (c.neg[p][i >> 5] >> (i & 31)) & 1u ? -v : v;
}

// The normalised Walsh-Hadamard transform of the block's row (reference
// src/kv_quant/scalar.rs:27-47); `finite` is the same in every thread.
__device__ __forceinline__ float kvq_hadamard(float v, float *sh, bool &finite) {
  const int i = threadIdx.x;
#pragma unroll
  for (int half = 1; half < 32; half <<= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, v, half);
    v = (i & half) ? __fsub_rn(o, v) : __fadd_rn(v, o);
  }
#pragma unroll
  for (int half = 32; half < kKvqDim; half <<= 1) {
    sh[i] = v;
    __syncthreads();
    const float o = sh[i ^ half];
    __syncthreads();
    v = (i & half) ? __fsub_rn(o, v) : __fadd_rn(v, o);
  }
  v = __fmul_rn(v, 0.0625f);
  finite = __syncthreads_and(is_finite_f(v));
  return v;
}

// Quantizer::rotate / forward (reference src/kv_quant.rs:479-488, 831-848).
__device__ __forceinline__ float kvq_forward(const KvqCodec &c, float v, float *sh, bool &finite) {
  finite = true;
  for (int p = 0; p < 3 && finite; ++p) v = kvq_hadamard(kvq_sign(c, p, threadIdx.x, v), sh, finite);
  return v;
}

// Quantizer::inverse (reference src/kv_quant.rs:490-525).
__device__ __forceinline__ float kvq_inverse(const KvqCodec &c, float v, float *sh, bool &finite) {
  finite = true;
  for (int p = 2; p >= 0 && finite; --p) v = kvq_sign(c, p, threadIdx.x, kvq_hadamard(v, sh, finite));
  return v;
}

struct KvqEncodeSmem {
  float row[kKvqDim];
  float sh[kKvqDim];
  double a[kKvqDim], b[kKvqDim];
  uint8_t code[kKvqDim];
  double sq;
  float scale;
};

// Quantizer::encode (reference src/kv_quant.rs:515-565; fitted scale
// src/kv_quant/fitted_scale.rs:8-48): thread i holds channel i of the row.
// Writes the record (when `rec` is set) and returns 0, or returns the status
// bit of the failure and writes nothing.  Every return is block-uniform.
__device__ unsigned kvq_encode_row(float x, const KvqCodec &c, uint8_t *rec, KvqEncodeSmem &sm) {
  const int i = threadIdx.x;
  const int nlev = c.bits == 3 ? 8 : 16;
  sm.row[i] = x;
  if (!__syncthreads_and(is_finite_f(x))) return kStatusInvalid;
  if (i == 0) {
    double s = 0.0;
    for (int j = 0; j < kKvqDim; ++j) s = __fma_rn((double)sm.row[j], (double)sm.row[j], s);
    sm.sq = s;
  }
  __syncthreads();
  const double sq = sm.sq;
  const int nbytes = kvq_record_bytes(c.bits);
  if (sq == 0.0) {  // the canonical zero record
    if (rec)
      for (int j = i; j < nbytes; j += kKvqDim) rec[j] = 0;
    return 0;
  }
  const float scale = __double2float_rn(__ddiv_rn(__dsqrt_rn(sq), 16.0));
  if (!is_finite_f(scale)) return kStatusNonfinite;
  if (scale == 0.0f) return kStatusInvalid;
  float v = __double2float_rn(__ddiv_rn((double)x, (double)scale));
  if (!__syncthreads_and(is_finite_f(v))) return kStatusNonfinite;
  bool finite;
  v = kvq_forward(c, v, sm.sh, finite);
  if (!finite) return kStatusNonfinite;
  // nearest level, the first code on ties (src/kv_quant/scalar.rs:49-61)
  int code = 0;
  float dist = fabsf(__fsub_rn(v, kvq_level(c.bits, 0)));
  for (int k = 1; k < nlev; ++k) {
    const float d = fabsf(__fsub_rn(v, kvq_level(c.bits, k)));
    if (d < dist) {
      code = k;
      dist = d;
    }
  }
  const float level = kvq_level(c.bits, code);
  if (!__syncthreads_and(is_finite_f(__fmul_rn(scale, level)))) return kStatusNonfinite;
  sm.code[i] = (uint8_t)code;
  float stored = scale;
  if (c.version == 2) {
    // the least-squares candidate, then the rotated-error guard
    sm.a[i] = (double)v;
    sm.b[i] = (double)level;
    __syncthreads();
    if (i == 0) {
      double cross = 0.0, energy = 0.0;
      for (int j = 0; j < kKvqDim; ++j) {
        cross = __fma_rn(sm.a[j], sm.b[j], cross);
        energy = __fma_rn(sm.b[j], sm.b[j], energy);
      }
      sm.scale = __double2float_rn(__dmul_rn((double)scale, __ddiv_rn(cross, energy)));
    }
    __syncthreads();
    const float cand = sm.scale;
    if (is_finite_f(cand) && cand > 0.0f && __float_as_uint(cand) != __float_as_uint(scale)) {
      const float recon = __fmul_rn(cand, level);
      const bool usable = __syncthreads_and(is_finite_f(recon));
      if (usable) {
        const double target = __dmul_rn((double)v, (double)scale);
        sm.a[i] = __dsub_rn(target, (double)__fmul_rn(scale, level));
        sm.b[i] = __dsub_rn(target, (double)recon);
        __syncthreads();
        if (i == 0) {
          double base = 0.0, fit = 0.0;
          for (int j = 0; j < kKvqDim; ++j) {
            base = __fma_rn(sm.a[j], sm.a[j], base);
            fit = __fma_rn(sm.b[j], sm.b[j], fit);
          }
          sm.scale = fit < base ? cand : scale;
        }
        __syncthreads();
        stored = sm.scale;
      }
    }
  }
  __syncthreads();
  if (rec) {
    if (i < c.bits * 32) {
      // byte i of the code stream: bits 8i..8i+7, code j at bits j*bits..
      unsigned byte = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int sb = 8 * i + k;
        byte |= ((sm.code[sb / c.bits] >> (sb % c.bits)) & 1u) << k;
      }
      rec[4 + i] = (uint8_t)byte;
    }
    if (i == 0) *reinterpret_cast<uint32_t *>(rec) = __float_as_uint(stored);
  }
  return 0;
}

// Record validity (reference src/kv_quant.rs:850-866): a finite, non-negative
// scale (not -0), and all-zero codes when it is +0.
__device__ __forceinline__ bool kvq_scale_ok(uint32_t sbits) {
  const float s = __uint_as_float(sbits);
  return is_finite_f(s) && !(sbits >> 31);
}

// ---- codec kernels (one block of 256 threads per row) ------------------

__global__ void __launch_bounds__(kKvqDim) kvq_encode_kernel(KvqCodec c, const float *rows,
                                                             uint8_t *records, unsigned *status) {
  __shared__ KvqEncodeSmem sm;
  grid_dependency_wait();
  grid_dependents_launch();
  const long r = blockIdx.x;
  const unsigned bad = kvq_encode_row(rows[r * kKvqDim + threadIdx.x], c,
                                      records + r * kvq_record_bytes(c.bits), sm);
  if (bad && threadIdx.x == 0) report(status, bad);
}

// Quantizer::decode (reference src/kv_quant.rs:812-822): accumulate with
// weight 1 into zeros, then the inverse rotation.
__global__ void __launch_bounds__(kKvqDim) kvq_decode_kernel(KvqCodec c, const uint8_t *records,
                                                             float *rows, unsigned *status) {
  __shared__ float sh[kKvqDim];
  grid_dependency_wait();
  grid_dependents_launch();
  const int i = threadIdx.x;
  const uint8_t *rec = records + (long)blockIdx.x * kvq_record_bytes(c.bits);
  const uint32_t sbits = *reinterpret_cast<const uint32_t *>(rec);
  const float scale = __uint_as_float(sbits);
  const int off = i * c.bits;
  unsigned code = rec[4 + off / 8] >> (off % 8);
  if (off % 8 + c.bits > 8) code |= (unsigned)rec[4 + off / 8 + 1] << (8 - off % 8);
  code &= (1u << c.bits) - 1u;
  const bool ok = __syncthreads_and(kvq_scale_ok(sbits) && (scale != 0.0f || code == 0));
  if (!ok) {
    if (i == 0) report(status, kStatusInvalid);
    return;
  }
  float v = 0.0f;
  if (scale != 0.0f) v = __fadd_rn(0.0f, __fmul_rn(__fmul_rn(1.0f, scale), kvq_level(c.bits, code)));
  if (!__syncthreads_and(is_finite_f(v))) {
    if (i == 0) report(status, kStatusNonfinite);
    return;
  }
  bool finite;
  v = kvq_inverse(c, v, sh, finite);
  if (!finite) {
    if (i == 0) report(status, kStatusNonfinite);
    return;
  }
  rows[(long)blockIdx.x * kKvqDim + i] = v;
}

// RoPE (cos, sin) pair i of position `pos` (reference src/graph.rs:6406-6437,
// as attention_decode_kernel forms it): angle = pos * theta_scale^i by i
// repeated binary32 multiplications, position 0 past 3 * section.
__device__ __forceinline__ void kvq_rope_pair(int i, int pos, float theta_scale,
                                              const int *sections, float *cs) {
  float theta = (float)pos;
  for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, theta_scale);
  const float angle = i < 3 * sections[i % 3] ? theta : 0.0f;
  cs[2 * i] = cos_cr(angle);
  cs[2 * i + 1] = sin_cr(angle);
}

// The model step's append: the current position's key (RMSNorm, RoPE,
// binary16 rounding) and value (binary16 rounding) of every KV head, encoded
// into the caches at *position (reference src/graph.rs:4521-4540 and
// src/graph/quantized_kv.rs:629-657 prepare_current).  Grid: 2 * kv_heads
// blocks, keys first.
struct KvqAppendArgs {
  KvqCodec kc, vc;
  int kv_heads, rope_dim, sections[3];
  float eps, theta_scale;
  const float *key_in, *value_in;  // [kv_heads][256]
  const float *k_norm;
  uint8_t *kcache, *vcache;        // [context][kv_heads][record]
  const int *position;
  unsigned *status;
};

__global__ void __launch_bounds__(kKvqDim) kvq_append_kernel(KvqAppendArgs a) {
  __shared__ KvqEncodeSmem sm;
  __shared__ float cs[64], buf[kKvqDim];
  __shared__ double red[kKvqDim / 32];
  const int i = threadIdx.x;
  const bool value = (int)blockIdx.x >= a.kv_heads;
  const int kvh = value ? blockIdx.x - a.kv_heads : blockIdx.x;
  const int pos = *a.position;
  if (i < a.rope_dim / 2) kvq_rope_pair(i, pos, a.theta_scale, a.sections, cs);
  grid_dependency_wait();
  grid_dependents_launch();
  __syncthreads();
  float x;
  if (value)
    x = round_f16(a.value_in[kvh * kKvqDim + i]);
  else
    x = norm_rope_round(a.key_in + (long)kvh * kKvqDim, a.k_norm, a.eps, kKvqDim, a.rope_dim, cs,
                        buf, red);
  const KvqCodec &c = value ? a.vc : a.kc;
  uint8_t *rec = (value ? a.vcache : a.kcache) +
                 ((size_t)pos * a.kv_heads + kvh) * kvq_record_bytes(c.bits);
  const unsigned bad = kvq_encode_row(x, c, rec, sm);
  if (bad && i == 0) report(a.status, bad);
}

// ---- attention over records --------------------------------------------

struct KvqAttnArgs {
  KvqCodec kc, vc;              // key codec (4 bits), value codec
  int heads, kv_heads;
  // the query: RMSNorm * q_norm, RoPE and binary16 rounding of the first
  // half of projected[h] when `projected` is set (the model step), else the
  // rows query[h]
  const float *projected;       // [heads][2][256]: query then gate
  const float *q_norm;
  float eps, theta_scale;
  int rope_dim, sections[3];
  const float *query;           // [heads][256]
  const float *gate;            // gate row of head h: gate + h * gate_stride
  long gate_stride;
  const uint8_t *keys, *values; // [positions][kv_heads][record]
  const int *position;          // n = *position + 1 when set, else n_fixed
  int n_fixed;
  float attn_scale;
  float *out;                   // [heads][256]
  unsigned *status;
};

// Dynamic shared memory of a kvq_attend_kernel launch serving up to `cap`
// positions: the score row, then two value staging buffers.
__host__ __device__ constexpr size_t kvq_attend_smem(int cap) {
  return ((size_t)cap * 4 + 15) / 16 * 16 + 2 * (size_t)kKvqChunk * 5 * 4;
}

__global__ void __launch_bounds__(kKvqDim) kvq_attend_kernel(KvqAttnArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float kvq_dyn[];
  __shared__ double qd[kKvqDim];
  __shared__ double levk[16];
  __shared__ float levv[16];
  __shared__ float sh[kKvqDim], cs[64], buf[kKvqDim];
  __shared__ float vout[32];
  __shared__ double red[kKvqDim / 32];
  __shared__ float fred[kKvqDim / 32];
  __shared__ float s_inv;
  const int i = threadIdx.x, warp = i >> 5, lane = i & 31;
  const int rank = (int)cluster.block_rank();
  const int h = blockIdx.x / kKvqSplit;
  const int kvh = h / (a.heads / a.kv_heads);
  if (i < 16) {
    levk[i] = (double)kvq_level(4, i);
    levv[i] = i < (1 << a.vc.bits) ? kvq_level(a.vc.bits, i) : 0.0f;
  }
  const int pos = a.position ? *a.position : 0;
  if (a.projected && i < a.rope_dim / 2) kvq_rope_pair(i, pos, a.theta_scale, a.sections, cs);
  grid_dependency_wait();
  grid_dependents_launch();
  __syncthreads();
  unsigned bad = 0;
  const int n = a.position ? pos + 1 : a.n_fixed;
  float q;
  if (a.projected)
    q = norm_rope_round(a.projected + (long)h * 2 * kKvqDim, a.q_norm, a.eps, kKvqDim,
                        a.rope_dim, cs, buf, red);
  else
    q = a.query[(long)h * kKvqDim + i];
  bool finite = __syncthreads_and(is_finite_f(q));
  if (!finite) bad |= kStatusInvalid;
  float rq = kvq_forward(a.kc, finite ? q : 0.0f, sh, finite);
  if (!finite) bad |= kStatusNonfinite;
  qd[i] = (double)rq;
  __syncthreads();

  // scores of this CTA's share of the positions: a position per thread,
  // four binary64 lanes over the 4-bit codes
  float *scores = kvq_dyn;
  const int share = (n + kKvqSplit - 1) / kKvqSplit;
  const int lo = min(n, rank * share), hi = min(n, lo + share);
  const int krb = kvq_record_bytes(4);
  for (int p = lo + i; p < hi; p += kKvqDim) {
    const uint32_t *rec = reinterpret_cast<const uint32_t *>(
        a.keys + ((size_t)p * a.kv_heads + kvh) * krb);
    const uint32_t sbits = __ldg(rec);
    const float scale = __uint_as_float(sbits);
    double l0 = 0.0, l1 = 0.0, l2 = 0.0, l3 = 0.0;
    uint32_t any = 0;
#pragma unroll 4
    for (int w = 0; w < 32; ++w) {
      const uint32_t word = __ldg(rec + 1 + w);
      any |= word;
      const double *qq = qd + 8 * w;
      l0 = __fma_rn(qq[0], levk[word & 15u], l0);
      l1 = __fma_rn(qq[1], levk[(word >> 4) & 15u], l1);
      l2 = __fma_rn(qq[2], levk[(word >> 8) & 15u], l2);
      l3 = __fma_rn(qq[3], levk[(word >> 12) & 15u], l3);
      l0 = __fma_rn(qq[4], levk[(word >> 16) & 15u], l0);
      l1 = __fma_rn(qq[5], levk[(word >> 20) & 15u], l1);
      l2 = __fma_rn(qq[6], levk[(word >> 24) & 15u], l2);
      l3 = __fma_rn(qq[7], levk[word >> 28], l3);
    }
    float s = 0.0f;
    if (!kvq_scale_ok(sbits) || (scale == 0.0f && any)) {
      bad |= kStatusInvalid;
    } else if (scale != 0.0f) {
      const float unscaled = __double2float_rn(__dadd_rn(__dadd_rn(__dadd_rn(l0, l1), l2), l3));
      s = __fmul_rn(unscaled, scale);
      if (!is_finite_f(unscaled) || !is_finite_f(s)) bad |= kStatusNonfinite;
    }
    scores[p] = __fmul_rn(s, a.attn_scale);
  }
  cluster.sync();
  // every CTA gathers the other shares
  for (int r = 0; r < kKvqSplit; ++r) {
    if (r == rank) continue;
    const int rlo = min(n, r * share), rhi = min(n, rlo + share);
    const float *peer = cluster.map_shared_rank(scores, r);
    for (int p = rlo + i; p < rhi; p += kKvqDim) scores[p] = peer[p];
  }
  cluster.sync();  // no CTA rewrites its scores while a peer still reads them

  // softmax_round_f16 (reference src/kernels.rs softmax_round_f16): the
  // maximum, binary32 exponentials, their binary64 total in position order,
  // binary16-rounded probabilities
  float m = -INFINITY;
  for (int p = i; p < n; p += kKvqDim) m = fmaxf(m, scores[p]);
  m = block_max_f32(m, fred);
  if (!is_finite_f(m)) bad |= kStatusInvalid;
  for (int p = i; p < n; p += kKvqDim) scores[p] = exp_cr(__fsub_rn(scores[p], m));
  __syncthreads();
  if (i == 0) {
    double total = 0.0;
    int p = 0;
    for (; p + 4 <= n; p += 4) {
      const float4 e = *reinterpret_cast<const float4 *>(scores + p);
      total = __dadd_rn(total, (double)e.x);
      total = __dadd_rn(total, (double)e.y);
      total = __dadd_rn(total, (double)e.z);
      total = __dadd_rn(total, (double)e.w);
    }
    for (; p < n; ++p) total = __dadd_rn(total, (double)scores[p]);
    s_inv = __double2float_rn(__ddiv_rn(1.0, total));
  }
  __syncthreads();
  const float inv = s_inv;
  for (int p = i; p < n; p += kKvqDim) scores[p] = round_f16(__fmul_rn(scores[p], inv));

  // value scan over this CTA's 32 channels [32 rank, 32 rank + 32): warp 0
  // runs the chains, the other warps stage the next chunk's scales and code
  // slices (bits words per position)
  const int vb = a.vc.bits, vrb = kvq_record_bytes(vb);
  const int stride = 1 + vb;  // words per staged position
  uint32_t *stage = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(kvq_dyn) +
                                                 ((size_t)n * 4 + 15) / 16 * 16);
  const int nchunks = (n + kKvqChunk - 1) / kKvqChunk;
  auto stage_chunk = [&](int ck, int t0, int nt) {
    uint32_t *dst = stage + (size_t)(ck & 1) * kKvqChunk * 5;
    const int p0 = ck * kKvqChunk, cnt = min(kKvqChunk, n - p0);
    for (int e = t0; e < cnt * stride; e += nt) {
      const int pp = e / stride, w = e % stride;
      const uint32_t *rec = reinterpret_cast<const uint32_t *>(
          a.values + ((size_t)(p0 + pp) * a.kv_heads + kvh) * vrb);
      dst[e] = __ldg(rec + (w == 0 ? 0 : 1 + rank * vb + (w - 1)));
    }
  };
  stage_chunk(0, i, kKvqDim);
  __syncthreads();
  // the lane's code: bits [vb * lane, vb * lane + vb) of the slice
  const int cbit = vb * lane, cw = cbit >> 5, cs_ = cbit & 31;
  float acc = 0.0f;
  for (int ck = 0; ck < nchunks; ++ck) {
    if (warp != 0) {
      if (ck + 1 < nchunks) stage_chunk(ck + 1, i - 32, kKvqDim - 32);
    } else {
      const uint32_t *src = stage + (size_t)(ck & 1) * kKvqChunk * 5;
      const int p0 = ck * kKvqChunk, cnt = min(kKvqChunk, n - p0);
#pragma unroll 4
      for (int pp = 0; pp < cnt; ++pp) {
        const uint32_t *e = src + pp * stride;
        const uint32_t sbits = e[0];
        const float scale = __uint_as_float(sbits);
        uint32_t code = e[1 + cw] >> cs_;
        if (cs_ + vb > 32) code |= e[2 + cw] << (32 - cs_);
        code &= (1u << vb) - 1u;
        const uint32_t any = __ballot_sync(0xffffffffu, code != 0);
        const float ws = __fmul_rn(scores[p0 + pp], scale);
        if (!kvq_scale_ok(sbits) || (scale == 0.0f && any)) bad |= kStatusInvalid;
        if (!is_finite_f(ws)) bad |= kStatusNonfinite;
        acc = __fadd_rn(acc, __fmul_rn(ws, levv[code]));
      }
    }
    __syncthreads();
  }
  if (warp == 0) vout[lane] = acc;
  cluster.sync();
  float v = cluster.map_shared_rank(vout, i >> 5)[i & 31];
  if (!__syncthreads_and(is_finite_f(v))) bad |= kStatusNonfinite;
  v = kvq_inverse(a.vc, is_finite_f(v) ? v : 0.0f, sh, finite);
  if (!finite) bad |= kStatusNonfinite;
  if ((i >> 5) == rank) {
    const float o = __fmul_rn(v, sigmoid_f(a.gate[(long)h * a.gate_stride + i]));
    if (!is_finite_f(o)) bad |= kStatusNonfinite;
    a.out[(long)h * kKvqDim + i] = o;
  }
  if (bad) report(a.status, bad);
  cluster.sync();  // peers' shared memory stays live until every read is done
}

// One 8-CTA cluster per query head; `cap` bounds the positions served.
inline cudaError_t launch_kvq_attend(const KvqAttnArgs &a, int cap, cudaStream_t s, bool pdl) {
  const size_t smem = kvq_attend_smem(cap);
  cudaError_t e = cudaFuncSetAttribute(kvq_attend_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute cattr[2];
  cudaLaunchConfig_t cfg =
      pdl_config(dim3(a.heads * kKvqSplit), dim3(kKvqDim), smem, s, cattr, pdl);
  cattr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
  cattr[cfg.numAttrs].val.clusterDim.x = kKvqSplit;
  cattr[cfg.numAttrs].val.clusterDim.y = 1;
  cattr[cfg.numAttrs].val.clusterDim.z = 1;
  cfg.numAttrs += 1;
  return cudaLaunchKernelEx(&cfg, kvq_attend_kernel, a);
}

}  // namespace prism

// ---- C ABI: the codec and the attention over records -------------------
// The reference's codec API (src/kv_quant.rs Quantizer::encode / decode and
// src/graph/quantized_kv.rs attend_head) over arrays of rows.  Host
// variants copy in, run on the executor's stream and return the status;
// _device variants only enqueue.

namespace prism {

inline int kvq_codec_check(prism_b200_executor *ex, uint32_t bits, uint32_t version) {
  if (bits != 3 && bits != 4) return ex->fail(PRISM_B200_E_INVALID, "codec bits %u", bits);
  if (version != 1 && version != 2)
    return ex->fail(PRISM_B200_E_INVALID, "codec version %u", version);
  return PRISM_B200_OK;
}

// The policy's codecs: keys 4 bits; values 4 bits (rsq4), 4 bits fitted
// (rsq4vf) or 3 bits (rsq4k3v).
inline bool kvq_policy_codecs(uint32_t policy, KvqCodec *kc, KvqCodec *vc) {
  if (policy < PRISM_B200_KV_RSQ4 || policy > PRISM_B200_KV_RSQ4K3V) return false;
  *kc = kvq_codec(4, kKvqKeySeed, 1);
  *vc = kvq_codec(policy == PRISM_B200_KV_RSQ4K3V ? 3 : 4, kKvqValueSeed,
                  policy == PRISM_B200_KV_RSQ4VF ? 2 : 1);
  return true;
}

inline int kvq_attend_check(prism_b200_executor *ex, uint32_t policy, size_t positions,
                            uint32_t heads, uint32_t kv_heads, float attn_scale) {
  if (policy < PRISM_B200_KV_RSQ4 || policy > PRISM_B200_KV_RSQ4K3V)
    return ex->fail(PRISM_B200_E_INVALID, "KV policy %u has no rotated records", policy);
  if (positions == 0 || positions > (size_t)kKvqMaxPos)
    return ex->fail(positions ? PRISM_B200_E_UNSUPPORTED : PRISM_B200_E_INVALID,
                    "%zu positions (1..%d served)", positions, kKvqMaxPos);
  if (heads == 0 || kv_heads == 0 || heads % kv_heads || heads > 65535u / kKvqSplit)
    return ex->fail(PRISM_B200_E_INVALID, "%u query heads over %u KV heads", heads, kv_heads);
  if (!std::isfinite(attn_scale)) return ex->fail(PRISM_B200_E_INVALID, "attention scale");
  return PRISM_B200_OK;
}

inline cudaError_t kvq_enqueue_attend(prism_b200_executor *ex, uint32_t policy,
                                      const float *queries, const uint8_t *keys,
                                      const uint8_t *values, size_t positions, uint32_t heads,
                                      uint32_t kv_heads, float attn_scale, const float *gates,
                                      float *out, cudaStream_t s) {
  KvqAttnArgs a{};
  kvq_policy_codecs(policy, &a.kc, &a.vc);
  a.heads = (int)heads;
  a.kv_heads = (int)kv_heads;
  a.query = queries;
  a.gate = gates;
  a.gate_stride = kKvqDim;
  a.keys = keys;
  a.values = values;
  a.n_fixed = (int)positions;
  a.attn_scale = attn_scale;
  a.out = out;
  a.status = ex->d_status;
  return launch_kvq_attend(a, (int)positions, s, ex->pdl);
}

inline cudaError_t kvq_enqueue_encode(prism_b200_executor *ex, const KvqCodec &c,
                                      const float *rows, size_t n, uint8_t *records,
                                      cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)n), dim3(kKvqDim), 0, s, attr, ex->pdl);
  return cudaLaunchKernelEx(&cfg, kvq_encode_kernel, c, rows, records, ex->d_status);
}

}  // namespace prism

extern "C" {

int prism_b200_kvq_record_bytes(uint32_t bits) { return prism::kvq_record_bytes((int)bits); }

int prism_b200_kvq_encode_device(prism_b200_executor *ex, uint32_t bits, uint64_t seed,
                                 uint32_t version, const float *rows, size_t n,
                                 uint8_t *records, void *stream) {
  using namespace prism;
  int st = check_open(ex);
  if (st) return st;
  if ((st = kvq_codec_check(ex, bits, version))) return st;
  if (n == 0 || n > 0x7fffffffu || !rows || !records)
    return ex->fail(PRISM_B200_E_INVALID, "encode of %zu rows", n);
  cudaSetDevice(ex->device);
  CK(kvq_enqueue_encode(ex, kvq_codec((int)bits, seed, (int)version), rows, n, records,
                        pick(ex, stream)),
     "codec encode");
  return PRISM_B200_OK;
}

int prism_b200_kvq_encode(prism_b200_executor *ex, uint32_t bits, uint64_t seed, uint32_t version,
                          const float *rows, size_t n, uint8_t *records) {
  using namespace prism;
  int st = check_open(ex);
  if (st) return st;
  if ((st = kvq_codec_check(ex, bits, version))) return st;
  if (n == 0 || n > 0x7fffffffu || !rows || !records)
    return ex->fail(PRISM_B200_E_INVALID, "encode of %zu rows", n);
  cudaSetDevice(ex->device);
  const size_t rb = (size_t)kvq_record_bytes((int)bits);
  CK(ex->x.ensure(n * kKvqDim * 4), "codec rows");
  CK(ex->y.ensure(n * rb), "codec records");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->x.ptr, rows, n * kKvqDim * 4, cudaMemcpyHostToDevice, s), "rows in");
  CK(kvq_enqueue_encode(ex, kvq_codec((int)bits, seed, (int)version),
                        static_cast<const float *>(ex->x.ptr), n,
                        static_cast<uint8_t *>(ex->y.ptr), s),
     "codec encode");
  if ((st = finish(ex, s))) return st;
  CK(cudaMemcpyAsync(records, ex->y.ptr, n * rb, cudaMemcpyDeviceToHost, s), "records out");
  CK(cudaStreamSynchronize(s), "records out");
  return PRISM_B200_OK;
}

int prism_b200_kvq_decode(prism_b200_executor *ex, uint32_t bits, uint64_t seed,
                          const uint8_t *records, size_t n, float *rows) {
  using namespace prism;
  int st = check_open(ex);
  if (st) return st;
  if ((st = kvq_codec_check(ex, bits, 1))) return st;
  if (n == 0 || n > 0x7fffffffu || !rows || !records)
    return ex->fail(PRISM_B200_E_INVALID, "decode of %zu records", n);
  cudaSetDevice(ex->device);
  const size_t rb = (size_t)kvq_record_bytes((int)bits);
  CK(ex->x.ensure(n * kKvqDim * 4), "codec rows");
  CK(ex->y.ensure(n * rb), "codec records");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->y.ptr, records, n * rb, cudaMemcpyHostToDevice, s), "records in");
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)n), dim3(kKvqDim), 0, s, attr, ex->pdl);
  CK(cudaLaunchKernelEx(&cfg, kvq_decode_kernel, kvq_codec((int)bits, seed, 1),
                        static_cast<const uint8_t *>(ex->y.ptr), static_cast<float *>(ex->x.ptr),
                        ex->d_status),
     "codec decode");
  if ((st = finish(ex, s))) return st;
  CK(cudaMemcpyAsync(rows, ex->x.ptr, n * kKvqDim * 4, cudaMemcpyDeviceToHost, s), "rows out");
  CK(cudaStreamSynchronize(s), "rows out");
  return PRISM_B200_OK;
}

int prism_b200_kvq_attend_device(prism_b200_executor *ex, uint32_t policy, const float *queries,
                                 const uint8_t *keys, const uint8_t *values, size_t positions,
                                 uint32_t heads, uint32_t kv_heads, float attn_scale,
                                 const float *gates, float *out, void *stream) {
  using namespace prism;
  int st = check_open(ex);
  if (st) return st;
  if ((st = kvq_attend_check(ex, policy, positions, heads, kv_heads, attn_scale))) return st;
  if (!queries || !keys || !values || !gates || !out)
    return ex->fail(PRISM_B200_E_INVALID, "null attention buffer");
  cudaSetDevice(ex->device);
  CK(kvq_enqueue_attend(ex, policy, queries, keys, values, positions, heads, kv_heads,
                        attn_scale, gates, out, pick(ex, stream)),
     "rotated attention");
  return PRISM_B200_OK;
}

int prism_b200_kvq_attend(prism_b200_executor *ex, uint32_t policy, const float *queries,
                          const uint8_t *keys, const uint8_t *values, size_t positions,
                          uint32_t heads, uint32_t kv_heads, float attn_scale, const float *gates,
                          float *out) {
  using namespace prism;
  int st = check_open(ex);
  if (st) return st;
  if ((st = kvq_attend_check(ex, policy, positions, heads, kv_heads, attn_scale))) return st;
  if (!queries || !keys || !values || !gates || !out)
    return ex->fail(PRISM_B200_E_INVALID, "null attention buffer");
  cudaSetDevice(ex->device);
  const size_t kb = (size_t)kvq_record_bytes(4) * kv_heads * positions;
  const size_t vb = (size_t)kvq_record_bytes(policy == PRISM_B200_KV_RSQ4K3V ? 3 : 4) *
                    kv_heads * positions;
  const size_t rows = (size_t)heads * kKvqDim * 4;
  CK(ex->x.ensure(2 * rows), "attention rows");  // queries, then gates
  CK(ex->y.ensure(rows), "attention output");
  CK(ex->ints.ensure(kb), "key records");
  CK(ex->ints2.ensure(vb), "value records");
  cudaStream_t s = ex->stream;
  uint8_t *xq = static_cast<uint8_t *>(ex->x.ptr);
  CK(cudaMemcpyAsync(xq, queries, rows, cudaMemcpyHostToDevice, s), "queries in");
  CK(cudaMemcpyAsync(xq + rows, gates, rows, cudaMemcpyHostToDevice, s), "gates in");
  CK(cudaMemcpyAsync(ex->ints.ptr, keys, kb, cudaMemcpyHostToDevice, s), "keys in");
  CK(cudaMemcpyAsync(ex->ints2.ptr, values, vb, cudaMemcpyHostToDevice, s), "values in");
  CK(kvq_enqueue_attend(ex, policy, reinterpret_cast<const float *>(xq),
                        static_cast<const uint8_t *>(ex->ints.ptr),
                        static_cast<const uint8_t *>(ex->ints2.ptr), positions, heads, kv_heads,
                        attn_scale, reinterpret_cast<const float *>(xq + rows),
                        static_cast<float *>(ex->y.ptr), s),
     "rotated attention");
  if ((st = finish(ex, s))) return st;
  CK(cudaMemcpyAsync(out, ex->y.ptr, rows, cudaMemcpyDeviceToHost, s), "output out");
  CK(cudaStreamSynchronize(s), "output out");
  return PRISM_B200_OK;
}

}  // extern "C"
