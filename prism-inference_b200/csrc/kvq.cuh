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
#include "flow.cuh"  // cp_async4, cp_async_commit, cp_async_wait_*
#include "model_kernels.cuh"

namespace prism {

constexpr int kKvqDim = 256;
constexpr int kKvqSplit = 8;        // CTAs (one cluster) per query head
constexpr int kKvqMaxPos = 32768;   // positions one attention launch serves
constexpr int kKvqChunk = 128;      // value-scan staging chunk, positions
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
__device__ __forceinline__ float kvq_forward(const KvqCodec &c, float v, float *sh,
                                             bool &finite) {
  finite = true;
  for (int p = 0; p < 3 && finite; ++p)
    v = kvq_hadamard(kvq_sign(c, p, threadIdx.x, v), sh, finite);
  return v;
}

// Quantizer::inverse (reference src/kv_quant.rs:490-525).
__device__ __forceinline__ float kvq_inverse(const KvqCodec &c, float v, float *sh,
                                             bool &finite) {
  finite = true;
  for (int p = 2; p >= 0 && finite; --p)
    v = kvq_sign(c, p, threadIdx.x, kvq_hadamard(v, sh, finite));
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
__device__ unsigned kvq_encode_row(float x, const KvqCodec &c, uint8_t *rec,
                                   KvqEncodeSmem &sm) {
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
  // optional timeline (CTA 0): [0] start, [1] query rotated, [2] scores,
  // [3] scores gathered, [4] softmax total, [5] value scan done, [6]/[7] exit
  unsigned long long *trace;
};

// Shared memory of kvq_attend_kernel: the score row (`cap` positions,
// padded to 16 B), then a region the phases take in turn -- two buffers of
// staged key records during the scores; during the value scan its ring of
// raw value words (per chunk: the scales, then 16-byte code slices) and two
// chunks of increments ([position][channel], rows of 36 words).
constexpr int kKvqKeyChunk = 224;  // key records per staging buffer
constexpr int kKvqRing = 8;        // raw value chunks: 6 in flight, 1 forming, 1 free
constexpr int kKvqIncRow = 36;     // words per position row of increments
constexpr size_t kKvqKeyBytes = (size_t)2 * kKvqKeyChunk * 33 * 4;
constexpr size_t kKvqRawChunk = (size_t)kKvqChunk * 5 * 4;  // scales + slices
constexpr size_t kKvqRawBytes = (size_t)kKvqRing * kKvqRawChunk;
constexpr size_t kKvqIncBytes = (size_t)2 * kKvqChunk * kKvqIncRow * 4;
constexpr size_t kKvqUnionBytes =
    kKvqKeyBytes > kKvqRawBytes + kKvqIncBytes ? kKvqKeyBytes : kKvqRawBytes + kKvqIncBytes;

__host__ __device__ constexpr size_t kvq_score_bytes(int cap) {
  return ((size_t)cap * 4 + 15) / 16 * 16;
}
__host__ __device__ constexpr size_t kvq_attend_smem(int cap) {
  return kvq_score_bytes(cap) + kKvqUnionBytes;
}

// Head h of the cluster's 8 CTAs.  Each CTA scores a contiguous share of the
// positions (a thread per position over the share's key records, staged by
// asynchronous copies), the CTAs exchange their maxima, exponentiate their
// shares and gather every share's exponentials; each then forms the total,
// the binary16 probabilities and the value chains of its 32 channels, and
// all 8 rebuild the inverse rotation of the 256.  VB: value code bits.
template <int VB>
__global__ void __launch_bounds__(kKvqDim) kvq_attend_kernel(KvqAttnArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float kvq_dyn[];
  __shared__ __align__(16) double qd[kKvqDim];
  __shared__ double levk[16];
  __shared__ float levv[16];
  __shared__ float sh[kKvqDim], cs[64], buf[kKvqDim];
  __shared__ float vout[32];
  __shared__ double red[kKvqDim / 32];
  __shared__ float fred[kKvqDim / 32];
  __shared__ float s_max, s_emin, s_inv;
  __shared__ double s_sum;
  const int i = threadIdx.x, warp = i >> 5, lane = i & 31;
  const int rank = (int)cluster.block_rank();
  const int h = blockIdx.x / kKvqSplit;
  const int kvh = h / (a.heads / a.kv_heads);
  trace_stamp(a.trace, 0);
  if (i < 16) {
    levk[i] = (double)kvq_level(4, i);
    levv[i] = i < (1 << VB) ? kvq_level(VB, i) : 0.0f;
  }
  const int pos = a.position ? *a.position : 0;
  if (a.projected && i < a.rope_dim / 2) kvq_rope_pair(i, pos, a.theta_scale, a.sections, cs);
  grid_dependency_wait();
  grid_dependents_launch();
  unsigned bad = 0;
  const int n = a.position ? pos + 1 : a.n_fixed;
  float *scores = kvq_dyn;
  uint8_t *ureg = reinterpret_cast<uint8_t *>(kvq_dyn) + kvq_score_bytes(n);
  // this CTA's share: a multiple of 4 positions (16-byte aligned rows)
  const int share = (n + 4 * kKvqSplit - 1) / (4 * kKvqSplit) * 4;
  const int lo = min(n, rank * share), hi = min(n, lo + share);
  const int krb = kvq_record_bytes(4);
  uint32_t *kst = reinterpret_cast<uint32_t *>(ureg);  // [2][chunk][33]
  const int nkc = (hi - lo + kKvqKeyChunk - 1) / kKvqKeyChunk;
  auto kfetch = [&](int c) {  // key records of chunk c into buffer c & 1
    if (c < nkc) {
      uint32_t *dst = kst + (size_t)(c & 1) * kKvqKeyChunk * 33;
      const int p0 = lo + c * kKvqKeyChunk, cnt = min(kKvqKeyChunk, hi - p0);
      for (int e = i; e < cnt * 33; e += kKvqDim) {
        const int pp = e / 33, w = e - pp * 33;
        cp_async4(dst + e, a.keys + ((size_t)(p0 + pp) * a.kv_heads + kvh) * krb + 4 * w);
      }
    }
    cp_async_commit();  // an empty group past the end keeps the count uniform
  };
  kfetch(0);
  kfetch(1);
  __syncthreads();
  float q;
  if (a.projected)
    q = norm_rope_round(a.projected + (long)h * 2 * kKvqDim, a.q_norm, a.eps, kKvqDim,
                        a.rope_dim, cs, buf, red);
  else
    q = a.query[(long)h * kKvqDim + i];
  bool finite = __syncthreads_and(is_finite_f(q));
  if (!finite) bad |= kStatusInvalid;
  const float rq = kvq_forward(a.kc, finite ? q : 0.0f, sh, finite);
  if (!finite) bad |= kStatusNonfinite;
  qd[i] = (double)rq;
  trace_stamp(a.trace, 1);

  // scores of the share, a position per thread: four binary64 lanes, each
  // adding the exact products q_i * level in channel order
  for (int c = 0; c < nkc; ++c) {
    cp_async_wait_pending(1);
    __syncthreads();  // chunk c's records (and, first, the query) visible
    const int p0 = lo + c * kKvqKeyChunk, cnt = min(kKvqKeyChunk, hi - p0);
    if (i < cnt) {
      const uint32_t *r = kst + (size_t)(c & 1) * kKvqKeyChunk * 33 + i * 33;
      const uint32_t sbits = r[0];
      const float scale = __uint_as_float(sbits);
      double l0 = 0.0, l1 = 0.0, l2 = 0.0, l3 = 0.0;
      uint32_t any = 0;
#pragma unroll 4
      for (int w = 0; w < 32; ++w) {
        const uint32_t word = r[1 + w];
        any |= word;
        const double2 *qq = reinterpret_cast<const double2 *>(qd + 8 * w);
        const double2 q01 = qq[0], q23 = qq[1], q45 = qq[2], q67 = qq[3];
        l0 = __fma_rn(q01.x, levk[word & 15u], l0);
        l1 = __fma_rn(q01.y, levk[(word >> 4) & 15u], l1);
        l2 = __fma_rn(q23.x, levk[(word >> 8) & 15u], l2);
        l3 = __fma_rn(q23.y, levk[(word >> 12) & 15u], l3);
        l0 = __fma_rn(q45.x, levk[(word >> 16) & 15u], l0);
        l1 = __fma_rn(q45.y, levk[(word >> 20) & 15u], l1);
        l2 = __fma_rn(q67.x, levk[(word >> 24) & 15u], l2);
        l3 = __fma_rn(q67.y, levk[word >> 28], l3);
      }
      float s = 0.0f;
      if (!kvq_scale_ok(sbits) || (scale == 0.0f && any)) {
        bad |= kStatusInvalid;
      } else if (scale != 0.0f) {
        const float unscaled =
            __double2float_rn(__dadd_rn(__dadd_rn(__dadd_rn(l0, l1), l2), l3));
        s = __fmul_rn(unscaled, scale);
        if (!is_finite_f(unscaled) || !is_finite_f(s)) bad |= kStatusNonfinite;
      }
      scores[p0 + i] = __fmul_rn(s, a.attn_scale);
    }
    __syncthreads();  // buffer c & 1 is free again
    kfetch(c + 2);
  }
  cp_async_wait_all();
  trace_stamp(a.trace, 2);

  // softmax_round_f16 (reference src/kernels.rs softmax_round_f16): the
  // maximum over every share first
  float m = -INFINITY;
  for (int p = lo + i; p < hi; p += kKvqDim) m = fmaxf(m, scores[p]);
  m = block_max_f32(m, fred);
  if (i == 0) s_max = m;
  cluster.sync();
  float M = -INFINITY;
  for (int r = 0; r < kKvqSplit; ++r) M = fmaxf(M, *cluster.map_shared_rank(&s_max, r));
  if (!is_finite_f(M)) bad |= kStatusInvalid;
  // the share's binary32 exponentials, their minimum and binary64 sum
  float emin = INFINITY;
  double part = 0.0;
  for (int p = lo + i; p < hi; p += kKvqDim) {
    const float e = exp_cr(__fsub_rn(scores[p], M));
    scores[p] = e;
    emin = fminf(emin, e);
    part = __dadd_rn(part, (double)e);
  }
  emin = -block_max_f32(-emin, fred);
  part = block_sum_f64(part, red);
  if (i == 0) {
    s_emin = emin;
    s_sum = part;
  }
  cluster.sync();
  // every share's exponentials into this CTA's row
  for (int r = 0; r < kKvqSplit; ++r) {
    if (r == rank) continue;
    const int rlo = min(n, r * share), rhi = min(n, rlo + share), n4 = (rhi - rlo) / 4;
    const float *peer = cluster.map_shared_rank(scores, r);
    for (int k = i; k < n4; k += kKvqDim)
      reinterpret_cast<float4 *>(scores + rlo)[k] = reinterpret_cast<const float4 *>(peer + rlo)[k];
    for (int p = rlo + 4 * n4 + i; p < rhi; p += kKvqDim) scores[p] = peer[p];
  }
  float gmin = INFINITY;
  double tree = 0.0;
  for (int r = 0; r < kKvqSplit; ++r) {
    gmin = fminf(gmin, *cluster.map_shared_rank(&s_emin, r));
    tree = __dadd_rn(tree, *cluster.map_shared_rank(&s_sum, r));
  }
  cluster.sync();  // every peer has its copy before anything is rewritten
  trace_stamp(a.trace, 3);
  // The total in position order.  When every exponential is at least
  // 2^(ceil(log2 n) - 30), all are multiples of the smallest one's ulp u and
  // the total stays below 2^53 u: every partial sum, in any order, is exact,
  // so the shares' tree is the sequential result.  Otherwise one thread adds
  // them in order.
  int lg = 0;
  while ((1 << lg) < n) ++lg;
  if (i == 0) {
    double total = tree;
    if (!(gmin >= ldexpf(1.0f, lg - 30))) {
      total = 0.0;
      int p = 0;
      for (; p + 4 <= n; p += 4) {
        const float4 e = *reinterpret_cast<const float4 *>(scores + p);
        total = __dadd_rn(total, (double)e.x);
        total = __dadd_rn(total, (double)e.y);
        total = __dadd_rn(total, (double)e.z);
        total = __dadd_rn(total, (double)e.w);
      }
      for (; p < n; ++p) total = __dadd_rn(total, (double)scores[p]);
    }
    s_inv = __double2float_rn(__ddiv_rn(1.0, total));
  }
  __syncthreads();
  const float inv = s_inv;
  trace_stamp(a.trace, 4);

  // value scan over this CTA's 32 channels [32 rank, 32 rank + 32).  Each
  // channel's binary32 chain runs in warp 0 in position order, one add per
  // position.  Warps 1-7 feed it: they copy the records' scales and code
  // slices into a ring by asynchronous copies, six chunks ahead, and form
  // the next chunk's increments round_f16(e * inv) * scale * level, a
  // position per thread, as rows of 36 words (the chain's lanes read one
  // row without bank conflicts, the formers' 16-byte stores spread over the
  // banks).  A chunk's tail up to a multiple of 8 positions holds +0, which
  // leaves a chain unchanged (its sum is never -0: it starts at +0 and
  // x + (-x) is +0).
  constexpr int kWords = 1 + VB;  // copies per position: the scale, the slice
  const int vrb = kvq_record_bytes(VB);
  uint8_t *raw = ureg;                                             // [ring] chunks
  float *inc = reinterpret_cast<float *>(ureg + kKvqRawBytes);     // [2][chunk][36]
  constexpr int kLead = kKvqRing - 2;
  const int nchunks = (n + kKvqChunk - 1) / kKvqChunk;
  const int pt = i - 32, np = kKvqDim - 32;  // producer index and count
  auto fetch = [&](int ck) {  // chunk ck into ring slot ck % kKvqRing
    if (ck < nchunks) {
      uint32_t *sc = reinterpret_cast<uint32_t *>(raw + (size_t)(ck % kKvqRing) * kKvqRawChunk);
      uint32_t *sl = sc + kKvqChunk;  // [chunk][4] slice words
      const int p0 = ck * kKvqChunk, cnt = min(kKvqChunk, n - p0);
      for (int e = pt; e < cnt * kWords; e += np) {
        const int pp = e / kWords, w = e - pp * kWords;
        const uint32_t *rec = reinterpret_cast<const uint32_t *>(
            a.values + ((size_t)(p0 + pp) * a.kv_heads + kvh) * vrb);
        if (w == 0)
          cp_async4(sc + pp, rec);
        else
          cp_async4(sl + 4 * pp + (w - 1), rec + 1 + rank * VB + (w - 1));
      }
    }
    cp_async_commit();
  };
  auto form = [&](int ck) {  // increments of chunk ck into slot ck & 1
    const uint32_t *sc =
        reinterpret_cast<const uint32_t *>(raw + (size_t)(ck % kKvqRing) * kKvqRawChunk);
    const uint4 *sl = reinterpret_cast<const uint4 *>(sc + kKvqChunk);
    float *dst = inc + (size_t)(ck & 1) * kKvqChunk * kKvqIncRow;
    const int p0 = ck * kKvqChunk, cnt = min(kKvqChunk, n - p0);
    const int cnt8 = (cnt + 7) & ~7;
    for (int pp = pt; pp < cnt8; pp += np) {
      float4 *row = reinterpret_cast<float4 *>(dst + pp * kKvqIncRow);
      if (pp >= cnt) {
#pragma unroll
        for (int j = 0; j < 8; ++j) row[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        continue;
      }
      const uint32_t sbits = sc[pp];
      const float scale = __uint_as_float(sbits);
      const uint4 wv = sl[pp];
      const uint64_t lo64 = (uint64_t)wv.x | ((uint64_t)wv.y << 32);
      const uint64_t hi64 = (uint64_t)wv.z | ((uint64_t)wv.w << 32);
      const float ws = __fmul_rn(round_f16(__fmul_rn(scores[p0 + pp], inv)), scale);
      const bool nonzero = (wv.x | wv.y | wv.z | (VB == 4 ? wv.w : 0u)) != 0u;
      if (!kvq_scale_ok(sbits) || (scale == 0.0f && nonzero)) bad |= kStatusInvalid;
      if (!is_finite_f(ws)) bad |= kStatusNonfinite;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int bit = VB * (4 * j + k);  // code 4j + k of the slice
          const uint32_t code =
              bit < 64 ? (uint32_t)(bit + VB <= 64 ? (lo64 >> bit)
                                                   : ((lo64 >> bit) | (hi64 << (64 - bit))))
                       : (uint32_t)(hi64 >> (bit - 64));
          v[k] = __fmul_rn(ws, levv[code & ((1u << VB) - 1u)]);
        }
        row[j] = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
  };
  if (warp != 0) {
    for (int ck = 0; ck <= kLead; ++ck) fetch(ck);
    cp_async_wait_pending(kLead);  // chunk 0 landed
  }
  __syncthreads();
  if (warp != 0) form(0);
  __syncthreads();
  float acc = 0.0f;
  for (int ck = 0; ck < nchunks; ++ck) {
    if (warp == 0) {
      const float *src = inc + (size_t)(ck & 1) * kKvqChunk * kKvqIncRow + lane;
      const int cnt8 = (min(kKvqChunk, n - ck * kKvqChunk) + 7) & ~7;
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = src[k * kKvqIncRow];
      for (int pp = 0; pp < cnt8; pp += 8) {
        const int nx = pp + 8 < cnt8 ? pp + 8 : pp;
        float w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = src[(nx + k) * kKvqIncRow];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = __fadd_rn(acc, v[k]);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = w[k];
      }
    } else if (ck + 1 < nchunks) {
      // chunk ck + 1 is the oldest pending group; the producers' barrier
      // publishes every thread's copies of it
      cp_async_wait_pending(kLead - 1);
      asm volatile("bar.sync 1, %0;" ::"r"(kKvqDim - 32) : "memory");
      form(ck + 1);
      fetch(ck + 1 + kLead);  // slot of chunk ck - 1, formed two iterations ago
    }
    __syncthreads();
  }
  if (warp != 0) cp_async_wait_all();
  trace_stamp(a.trace, 5);
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
  trace_exit(a.trace);
}

// One 8-CTA cluster per query head; `cap` bounds the positions served.
inline cudaError_t launch_kvq_attend(const KvqAttnArgs &a, int cap, cudaStream_t s, bool pdl) {
  const size_t smem = kvq_attend_smem(cap);
  auto kern = a.vc.bits == 3 ? kvq_attend_kernel<3> : kvq_attend_kernel<4>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute cattr[2];
  cudaLaunchConfig_t cfg =
      pdl_config(dim3(a.heads * kKvqSplit), dim3(kKvqDim), smem, s, cattr, pdl);
  cattr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
  cattr[cfg.numAttrs].val.clusterDim.x = kKvqSplit;
  cattr[cfg.numAttrs].val.clusterDim.y = 1;
  cattr[cfg.numAttrs].val.clusterDim.z = 1;
  cfg.numAttrs += 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
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
