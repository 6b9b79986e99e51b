// prefill.cuh -- batched prompt ingestion of one sequence.
//
// The reference ingests a prompt token by token through the decoder
// (src/lib.rs:229-247 Decoder::ingest) or through its tiled prefill
// (src/graph/prefill.rs), which shares each weight row across a tile of
// tokens.  Here all the prompt's tokens go through every layer together:
//   * projections are tensor-core GEMMs over the T tokens (gemm.cuh), with
//     the same per-row binary32 chains as the decode matvecs;
//   * each Gated DeltaNet layer forms every token's convolution, q/k norms,
//     decay and beta at once (gdn_token_inputs_kernel), then runs the exact
//     recurrence over the tokens with each state row held in one warp's
//     registers for the whole prompt (gdn_rows_scan_kernel) -- the decode
//     kernel's arithmetic, token after token;
//   * each attention layer first writes the T new K/V rows to the cache
//     (kv_rows_kernel), then every token attends over its own prefix
//     (attention_decode_kernel with one grid row per token, no writes).
// The state left behind -- KV rows, recurrent state, convolution history,
// position -- is bit for bit what T decode-path ingestion steps leave.
// Included once by prism_b200.cu, after batch.cuh.
#pragma once

#include "batch.cuh"

namespace prism {

constexpr int kPrefillChunk = 2048;  // tokens per batched pass

// ---- Gated DeltaNet over the prompt's tokens --------------------------------
//
// The decode step's per-token work splits into what does not depend on the
// recurrent state -- convolution + SiLU of every channel, L2 normalisation of
// the q and k groups, decay and beta of every head -- done for all tokens at
// once (gdn_token_inputs_kernel), and the state recurrence proper, a chain
// over the tokens for each state row (gdn_rows_scan_kernel).

struct GdnTokensArgs {
  int S, groups, values, conv_k, T, channels;
  float eps;
  const float *mixed;               // [T][channels] qkv projections, before conv
  const float *beta_in, *alpha_in;  // [T][values]
  const float *conv_w, *dt_bias, *ssm_a;
  const float *hist_in;             // [channels][k-1] history before token 0
  float *act;                       // [T][channels] conv + SiLU, q and k L2-normalised
  float *db;                        // [T][values][2] decay, beta
  float *state;                     // [values][S][S], updated in place
  float *o_pre;                     // [T][values * S] pre-norm outputs
  unsigned *status;
};

constexpr int kScanRows = 16;  // state rows (warps) per CTA of the scan

// grid (T, 2 * groups + values), S (= 128) threads: block y < groups is q
// group y, y < 2 * groups k group y - groups, else v head y - 2 * groups
// (whose thread 0 also forms the head's decay and beta).  run_gdn's
// arithmetic: taps in order, SiLU, then the binary64 sum of squares as a
// warp butterfly per 32 values with the partials added in warp order.
__global__ void __launch_bounds__(128) gdn_token_inputs_kernel(GdnTokensArgs a) {
  constexpr int S = 128;
  __shared__ double red[S / 32];
  const int t = blockIdx.x, y = blockIdx.y, j = threadIdx.x;
  const int kw = a.groups * S, hist = a.conv_k - 1;
  const int part = y < a.groups ? 0 : y < 2 * a.groups ? 1 : 2;
  const int ch = part == 0 ? y * S + j : part == 1 ? kw + (y - a.groups) * S + j
                                                   : 2 * kw + (y - 2 * a.groups) * S + j;
  const float *cj = a.conv_w + (long)ch * a.conv_k;
  float sum = 0.0f;
  for (int i = 0; i < hist; ++i) {
    const int tt = t - hist + i;  // the token whose input is tap i
    const float hv = tt >= 0 ? a.mixed[(long)tt * a.channels + ch]
                             : a.hist_in[(long)ch * hist + (t + i)];
    sum = __fadd_rn(sum, __fmul_rn(hv, cj[i]));
  }
  sum = __fadd_rn(sum, __fmul_rn(a.mixed[(long)t * a.channels + ch], cj[hist]));
  float act = silu_f(sum);
  if (part < 2) {
    const double w = warp_sum_f64((double)__fmul_rn(act, act));
    if ((j & 31) == 0) red[j >> 5] = w;
    __syncthreads();
    double tot = 0.0;
    for (int i = 0; i < S / 32; ++i) tot += red[i];
    act = __fmul_rn(act, __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)tot), a.eps)));
  } else if (j == 0) {
    const int h = y - 2 * a.groups;
    a.db[((long)t * a.values + h) * 2] =
        recurrent_decay_f(a.alpha_in[(long)t * a.values + h], a.dt_bias[h], a.ssm_a[h], a.status);
    a.db[((long)t * a.values + h) * 2 + 1] = sigmoid_f(a.beta_in[(long)t * a.values + h]);
  }
  a.act[(long)t * a.channels + ch] = act;
}

// One warp per state row of value head h, kScanRows rows of one head per
// CTA (grid values * S / kScanRows, 32 * kScanRows threads): each row stays
// in its warp's registers for the whole prompt, lane l owning columns
// 4l .. 4l+3.  Per token, run_gdn's row arithmetic in its order: decay, s.k
// (binary64 partials, warp butterfly), delta, update, s.q.  The tokens'
// q, k, v, decay and beta come through shared memory in chunks of
// kScanTokens, loaded cooperatively a chunk ahead.  s.q only feeds the
// output, so its lane partials wait in shared memory and at the chunk's end
// lane t forms token t's sum in the butterfly's association.  Outputs leave
// once per chunk, coalesced.
constexpr int kScanTokens = 32;

// The warp butterfly's sum of 32 lane values v[0..31] (lane l adds lane
// l^16, then l^8, ...), evaluated by one thread.
__device__ __forceinline__ double butterfly_sum32(const double (&v)[32]) {
  double s16[16], s8[8], s4[4];
#pragma unroll
  for (int b = 0; b < 16; ++b) s16[b] = v[b] + v[b + 16];
#pragma unroll
  for (int b = 0; b < 8; ++b) s8[b] = s16[b] + s16[b + 8];
#pragma unroll
  for (int b = 0; b < 4; ++b) s4[b] = s8[b] + s8[b + 4];
  return (s4[0] + s4[2]) + (s4[1] + s4[3]);
}

constexpr size_t gdn_scan_smem() {
  return (size_t)2 * kScanTokens * (2 * 128 + 2 * kScanRows + 2) * sizeof(float)  // inputs, outputs
         + (size_t)kScanRows * kScanTokens * 33 * sizeof(double);  // s.q lane partials
}

__global__ void __launch_bounds__(32 * kScanRows, 1) gdn_rows_scan_kernel(GdnTokensArgs a) {
  constexpr int S = 128, R = kScanRows, TC = kScanTokens, NT = 32 * R;
  extern __shared__ __align__(128) uint8_t smem[];
  float *qs = reinterpret_cast<float *>(smem);  // [2][TC][S]
  float *ks = qs + 2 * TC * S;                  // [2][TC][S]
  float *vs = ks + 2 * TC * S;                  // [2][TC][R]
  float *os = vs + 2 * TC * R;                  // [2][TC][R]
  float *ds = os + 2 * TC * R;                  // [2][TC][2] decay, beta
  // [R][TC][33]: each token's s.q lane partials, reduced at the chunk's end
  double *dqs = reinterpret_cast<double *>(ds + 2 * TC * 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * R, row = row0 + warp;  // h * S + r
  if (row0 >= a.values * S) return;
  const int h = row0 / S, kh = h % a.groups, kw = a.groups * S;
  float *srow = a.state + (long)row * S;
  float4 s = reinterpret_cast<const float4 *>(srow)[lane];
  const float oscale = __fdiv_rn(1.0f, __fsqrt_rn((float)S));
  const int nc = (a.T + TC - 1) / TC;
  // cooperative chunk loads: q and k as float4 (TC * S / 4 each), v as
  // float4 (TC * R / 4), decay and beta (TC pairs)
  constexpr int QV = TC * S / 4, VV = TC * R / 4;
  static_assert(QV % NT == 0, "q/k chunk split");
  float4 rq[QV / NT], rk[QV / NT], rv = make_float4(0.f, 0.f, 0.f, 0.f);
  float2 rd = make_float2(0.f, 0.f);
  auto load = [&](int c) {
    const int tb = c * TC;
#pragma unroll
    for (int i = 0; i < QV / NT; ++i) {
      const int e = tid + i * NT, t = tb + e / (S / 4), j = 4 * (e % (S / 4));
      const long o = (long)t * a.channels;
      rq[i] = t < a.T ? *reinterpret_cast<const float4 *>(a.act + o + kh * S + j)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      rk[i] = t < a.T ? *reinterpret_cast<const float4 *>(a.act + o + kw + kh * S + j)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid < VV) {
      const int t = tb + tid / (R / 4), j = 4 * (tid % (R / 4));
      rv = t < a.T ? *reinterpret_cast<const float4 *>(a.act + (long)t * a.channels + 2 * kw + row0 + j)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (tid < TC) {
      const int t = tb + tid;
      rd = t < a.T ? *reinterpret_cast<const float2 *>(a.db + ((long)t * a.values + h) * 2)
                   : make_float2(0.f, 0.f);
    }
  };
  auto store = [&](int b) {
#pragma unroll
    for (int i = 0; i < QV / NT; ++i) {
      const int e = tid + i * NT;
      reinterpret_cast<float4 *>(qs + b * TC * S)[e] = rq[i];
      reinterpret_cast<float4 *>(ks + b * TC * S)[e] = rk[i];
    }
    if (tid < VV) reinterpret_cast<float4 *>(vs + b * TC * R)[tid] = rv;
    if (tid < TC) reinterpret_cast<float2 *>(ds + b * TC * 2)[tid] = rd;
  };
  load(0);
  store(0);
  __syncthreads();
  double *dqw = dqs + (size_t)warp * TC * 33;
  for (int c = 0; c < nc; ++c) {
    const int b = c & 1, tb = c * TC, tn = min(TC, a.T - tb);
    if (c + 1 < nc) load(c + 1);  // in flight during this chunk's recurrence
    const float *qb = qs + b * TC * S, *kb = ks + b * TC * S;
    const float *vb = vs + b * TC * R, *db = ds + b * TC * 2;
    float *ob = os + b * TC * R;
    for (int tt = 0; tt < tn; ++tt) {
      const float4 kk = reinterpret_cast<const float4 *>(kb + tt * S)[lane];
      const float4 qq = reinterpret_cast<const float4 *>(qb + tt * S)[lane];
      const float vv = vb[tt * R + warp], decay = db[2 * tt], beta = db[2 * tt + 1];
      s.x = __fmul_rn(decay, s.x);
      s.y = __fmul_rn(decay, s.y);
      s.z = __fmul_rn(decay, s.z);
      s.w = __fmul_rn(decay, s.w);
      double dk = (double)__fmul_rn(s.x, kk.x) + (double)__fmul_rn(s.y, kk.y) +
                  (double)__fmul_rn(s.z, kk.z) + (double)__fmul_rn(s.w, kk.w);
      dk = warp_sum_f64(dk);
      const float delta = __fmul_rn(__fsub_rn(vv, (float)dk), beta);
      s.x = __fadd_rn(s.x, __fmul_rn(delta, kk.x));
      s.y = __fadd_rn(s.y, __fmul_rn(delta, kk.y));
      s.z = __fadd_rn(s.z, __fmul_rn(delta, kk.z));
      s.w = __fadd_rn(s.w, __fmul_rn(delta, kk.w));
      dqw[tt * 33 + lane] = (double)__fmul_rn(s.x, qq.x) + (double)__fmul_rn(s.y, qq.y) +
                            (double)__fmul_rn(s.z, qq.z) + (double)__fmul_rn(s.w, qq.w);
    }
    __syncwarp();
    // lane tt reduces token tt's s.q partials in the butterfly's association
    if (lane < tn) {
      double v[32];
#pragma unroll
      for (int l = 0; l < 32; ++l) v[l] = dqw[lane * 33 + l];
      ob[lane * R + warp] = __fmul_rn((float)butterfly_sum32(v), oscale);
    }
    __syncwarp();
    if (c + 1 < nc) store(b ^ 1);
    __syncthreads();  // the next chunk's inputs and this chunk's outputs are complete
    for (int e = tid; e < tn * R; e += NT)
      a.o_pre[(long)(tb + e / R) * a.values * S + row0 + e % R] = ob[e];
  }
  reinterpret_cast<float4 *>(srow)[lane] = s;
  // A non-finite state element stays non-finite at every later token (decay
  // times inf or NaN is inf or NaN, and adding to inf or NaN never gives a
  // finite value), so the final state's check equals the decode kernel's
  // check after every token.
  const bool finite = is_finite_f(s.x) && is_finite_f(s.y) && is_finite_f(s.z) && is_finite_f(s.w);
  if (!__all_sync(0xffffffffu, finite) && lane == 0) report(a.status, kStatusNonfinite);
}

// Convolution history after the prompt: each channel's last k-1 inputs
// (from the prompt's projections, or the history before it when the prompt
// is shorter).  One thread per channel; out may alias in (every read of a
// channel precedes its writes, in the same thread).
__global__ void conv_history_kernel(const float *mixed, const float *hist_in, float *hist_out,
                                    int channels, int hist, int T) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= channels || hist <= 0 || hist > 8) return;
  float nv[8];
  for (int i = 0; i < hist; ++i) {
    const int tt = T - hist + i;
    nv[i] = tt >= 0 ? mixed[(long)tt * channels + ch] : hist_in[(long)ch * hist + (T + i)];
  }
  for (int i = 0; i < hist; ++i) hist_out[(long)ch * hist + i] = nv[i];
}

// y = RMSNorm(o_h) * w * SiLU(z_h) per (token, head), a warp per head: the
// binary64 sum of squares as the decode out-projection's gated prologue
// forms it (four 32-value butterfly sums, added in order).  grid (T), up to
// 32 warps per CTA.
__global__ void gated_rows_kernel(const float *o_pre, const float *zgate, const float *norm_w,
                                  int values, int S, float eps, float *out) {
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  for (int h = threadIdx.x >> 5; h < values; h += (int)(blockDim.x >> 5)) {
    const long base = ((long)t * values + h) * S;
    const float *o = o_pre + base;
    double tot = 0.0;
    for (int qd = 0; qd < S / 32; ++qd) {
      const float val = o[32 * qd + lane];
      tot += warp_sum_f64((double)__fmul_rn(val, val));
    }
    const float mean = (float)(tot / (double)S);
    const float nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int qd = 0; qd < S / 32; ++qd) {
      const int i = 32 * qd + lane;
      const float normed = __fmul_rn(__fmul_rn(o[i], nscale), norm_w[i]);
      out[base + i] = __fmul_rn(normed, silu_f(zgate[base + i]));
    }
  }
}

// ---- attention: the prompt's K/V rows ---------------------------------------

// The K and V cache rows of tokens p0 .. p0+T-1, as attention_decode_kernel's
// writer CTA produces them (RMSNorm, RoPE and binary16 rounding of k; binary16
// rounding of v; binary16 bits or Q8_0 records).  grid (kv_heads, T), hd
// threads.
__global__ void __launch_bounds__(kAttnThreads) kv_rows_kernel(AttnArgs a, int p0) {
  __shared__ __align__(16) float cs[64];
  __shared__ float buf[kAttnThreads];
  __shared__ double red[kAttnThreads / 32];
  const int kvh = blockIdx.x, t = blockIdx.y, i = threadIdx.x;
  const int hd = a.hd, kvw = a.kv_heads * hd;
  const int pos = p0 + t;
  if (i < a.rope_dim / 2) {
    float theta = (float)pos;
    for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, a.theta_scale);
    const float angle = i < 3 * a.sections[i % 3] ? theta : 0.0f;
    cs[2 * i] = cos_cr(angle);
    cs[2 * i + 1] = sin_cr(angle);
  }
  __syncthreads();
  float kc = norm_rope_round(a.key_in + (long)t * kvw + (long)kvh * hd, a.k_norm, a.eps, hd,
                             a.rope_dim, cs, buf, red);
  float vc = round_f16(a.value_in[(long)t * kvw + kvh * hd + i]);
  if (a.q8) {
    const int rb = q8_0_record_bytes(hd);
    const long at = ((long)pos * a.kv_heads + kvh) * rb;
    q8_0_roundtrip(kc, reinterpret_cast<uint8_t *>(a.kcache) + at, hd, a.status);
    q8_0_roundtrip(vc, reinterpret_cast<uint8_t *>(a.vcache) + at, hd, a.status);
  } else {
    a.kcache[(long)pos * kvw + kvh * hd + i] = float_to_half_bits(kc);
    a.vcache[(long)pos * kvw + kvh * hd + i] = float_to_half_bits(vc);
  }
}

// ---- attention over the prompt ----------------------------------------------
//
// Token t of the prompt (position pos = p0 + t) attends over positions
// 0 .. pos-1 of the cache and its own row.  attention_decode_kernel's
// arithmetic for it is fixed by its 8-CTA split: scores are binary64 sums of
// binary32 products, 8 dimensions per lane then a warp butterfly; the
// softmax maximum is global, the exponentials' binary64 total is formed per
// CTA (rank r of 8 owns positions [r*per, (r+1)*per), per = ceil(pos/8)) as
// a 256-thread block sum and the ranks' totals are added in rank order; the
// probabilities are rounded to binary16; each rank's value sums run over its
// positions in order from -0.0 and are added in rank order.
// attention_prefill_kernel reproduces exactly that for kPfQueries (token,
// head) queries per CTA that share one KV head's rows, staged once per CTA:
//   * binary16 KV: a query and a key are binary16 values, so their binary32
//     product is exact (22 significant bits, no underflow) and equals the
//     binary64 product: each score is a chain of binary64 FMAs on operands
//     converted once, in the same leaf order and reduction tree;
//   * Q8_0 KV: dequantized keys carry up to 18 bits, so the binary32
//     product rounds: the products are formed in binary32 and widened.

constexpr int kPfQueries = 16;  // (token, head) queries per CTA
constexpr int kPfChunk = 32;    // positions per staged chunk
constexpr int kPfThreads = 512; // two threads per head dimension in the value pass

struct PrefillAttnArgs {
  AttnArgs a;       // geometry, norms, caches; projected/attended strides per token
  int p0, T, G, TQ; // first position, tokens, heads per KV head, tokens per CTA
  int context;      // scratch positions per query
  const float *qrows;  // [T][heads][hd] normalised, rotated, binary16-rounded queries
  const float *scur;   // [T][heads] score of each token's own row
  float *scratch;      // [CTAs][kPfQueries][context] scores, then probabilities
};

// Queries and own-row scores (attention_decode_kernel's prologue): grid
// (heads, T), hd (= kAttnThreads) threads.  Runs after kv_rows_kernel.
__global__ void __launch_bounds__(kAttnThreads) query_rows_kernel(AttnArgs a, int p0,
                                                                  float *qrows, float *scur) {
  __shared__ __align__(16) float cs[64];
  __shared__ float buf[kAttnThreads];
  __shared__ double red[kAttnThreads / 32];
  const int h = blockIdx.x, t = blockIdx.y, i = threadIdx.x;
  const int hd = a.hd, kvw = a.kv_heads * hd, kvh = h / (a.heads / a.kv_heads);
  const int pos = p0 + t;
  if (i < a.rope_dim / 2) {
    float theta = (float)pos;
    for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, a.theta_scale);
    const float angle = i < 3 * a.sections[i % 3] ? theta : 0.0f;
    cs[2 * i] = cos_cr(angle);
    cs[2 * i + 1] = sin_cr(angle);
  }
  __syncthreads();
  const float q = norm_rope_round(a.projected + (long)t * a.seq_proj + (long)h * 2 * hd, a.q_norm,
                                  a.eps, hd, a.rope_dim, cs, buf, red);
  float kc;
  if (a.q8) {
    const int rb = q8_0_record_bytes(hd);
    kc = q8_0_value(reinterpret_cast<const uint8_t *>(a.kcache) + ((long)pos * a.kv_heads + kvh) * rb,
                    hd, i);
  } else {
    kc = half_bits_to_float(a.kcache[(long)pos * kvw + kvh * hd + i]);
  }
  const double s = block_sum_f64((double)__fmul_rn(q, kc), red);
  qrows[((long)t * a.heads + h) * hd + i] = q;
  if (i == 0) scur[(long)t * a.heads + h] = __fmul_rn((float)s, __fdiv_rn(1.0f, __fsqrt_rn((float)hd)));
}

// Exact binary16 -> binary64 widening from the bit fields (normal numbers
// and zeros; the rare subnormal, infinite or NaN input goes through
// binary32).
__device__ __forceinline__ double f16_bits_to_f64(uint16_t hb) {
  const uint32_t e = (hb >> 10) & 31u, m = hb & 1023u, sgn = (uint32_t)(hb >> 15) << 31;
  if (e - 1u < 30u) return __hiloint2double((int)(sgn | ((e + 1008u) << 20) | (m << 10)), 0);
  if ((hb & 0x7fffu) == 0) return __hiloint2double((int)sgn, 0);
  return (double)half_bits_to_float(hb);
}

// Staged operand type and product chain of each KV format.  Rows arrive as
// raw cache bytes (bulk copies) and are widened once per CTA.
template <bool Q8>
struct PfOps {
  using T = double;
  static constexpr int kRowBytes = 512;  // 256 binary16 values
  __device__ static T widen_row(const uint8_t *row, int d) {
    return f16_bits_to_f64(reinterpret_cast<const uint16_t *>(row)[d]);
  }
  __device__ static T widen(float x) { return (double)x; }
  // first term, next term of a binary64 chain of (exact) binary32 products
  __device__ static double first(T x, T y) { return x * y; }
  __device__ static double next(T x, T y, double acc) { return fma(x, y, acc); }
};

template <>
struct PfOps<true> {
  using T = float;
  static constexpr int kRowBytes = q8_0_record_bytes(256);
  __device__ static T widen_row(const uint8_t *row, int d) { return q8_0_value(row, 256, d); }
  __device__ static T widen(float x) { return x; }
  __device__ static double first(T x, T y) { return (double)__fmul_rn(x, y); }
  __device__ static double next(T x, T y, double acc) { return acc + (double)__fmul_rn(x, y); }
};

template <bool Q8>
constexpr size_t prefill_attn_smem() {
  using T = typename PfOps<Q8>::T;
  return (size_t)256 * kPfQueries * sizeof(T)                 // queries [hd][Q]
         + (size_t)256 * (kPfChunk + 2) * sizeof(T)           // keys [hd][chunk+2] / values [chunk][hd]
         + (size_t)8 * kPfQueries * kPfChunk * 8              // score partial trees [8][Q][chunk]
         + (size_t)kPfChunk * kPfQueries * sizeof(T)          // probabilities [chunk][Q]
         + (size_t)2 * kPfChunk * PfOps<Q8>::kRowBytes;       // raw rows, two buffers
}


// grid (kv_heads, ceil(T / TQ)), kPfThreads threads; hd == 256, G * TQ <=
// kPfQueries.  Query qi = tl * G + g is token t0 + tl, head kvh * G + g.
// The K rows and then the V rows of positions 0 .. (last query's position)
// stream through two raw buffers in chunks of kPfChunk (bulk copies, one per
// row, issued two chunks ahead).  16 warps: the score pass splits the leaf
// groups and the query halves, the value pass the dimensions and the query
// halves.
template <bool Q8>
__global__ void __launch_bounds__(kPfThreads, 1) attention_prefill_kernel(PrefillAttnArgs pa) {
  using Ops = PfOps<Q8>;
  using T = typename Ops::T;
  constexpr int HD = 256, QN = kPfQueries, CH = kPfChunk, RB = Ops::kRowBytes;
  constexpr int CP = CH + 2;  // key row pitch: pairs stay 16-byte aligned
  extern __shared__ __align__(128) uint8_t smem[];
  T *qT = reinterpret_cast<T *>(smem);                            // [HD][QN]
  T *rows = qT + HD * QN;                                         // [HD][CP] / [CH][HD]
  double *Rs = reinterpret_cast<double *>(rows + HD * CP);       // [8][QN][CH]
  T *pd = reinterpret_cast<T *>(Rs + 8 * QN * CH);                // [CH][QN]
  uint8_t *raw = reinterpret_cast<uint8_t *>(pd + CH * QN);       // [2][CH][RB]
  double *W = Rs;  // softmax group totals [QN][8][8], between the passes
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int qpos[QN], qvalid[QN];
  __shared__ float qmax[QN], qM[QN], qinv[QN], qpcur[QN];
  __shared__ unsigned qmask[QN];
  __shared__ int qcnt[QN];
  const AttnArgs &a = pa.a;
  const int kvh = blockIdx.x, t0 = blockIdx.y * pa.TQ, G = pa.G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.y * gridDim.x + blockIdx.x;
  float *S = pa.scratch + (long)cta * QN * pa.context;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  if (tid < QN) {
    const int tl = tid / G, t = t0 + tl;
    const bool v = tid < G * pa.TQ && t < pa.T;
    qvalid[tid] = v;
    qpos[tid] = v ? pa.p0 + t : 0;
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init_fence();
  }
  // queries, transposed: qT[d][qi]
  for (int k = tid; k < HD * QN; k += kPfThreads) {
    const int qi = k / HD, d = k % HD, t = t0 + qi / G;
    const bool v = qi < G * pa.TQ && t < pa.T;
    const int h = kvh * G + qi % G;
    qT[d * QN + qi] = Ops::widen(v ? pa.qrows[((long)t * a.heads + h) * HD + d] : 0.0f);
  }
  __syncthreads();
  int plast = 0;
  for (int qi = 0; qi < QN; ++qi) plast = max(plast, qpos[qi]);
  const int nk = (plast + CH - 1) / CH;  // chunks per pass
  // chunk g of the sequence: K chunks 0..nk-1, then V chunks
  auto issue = [&](int g) {
    const bool v = g >= nk;
    const int c0 = (v ? g - nk : g) * CH, count = min(CH, plast - c0);
    uint64_t *bar = &bars[g & 1];
    if (lane == 0) mbar_arrive_expect_tx(bar, (unsigned)(count * RB));
    __syncwarp();
    if (lane < count) {
      const long p = c0 + lane;
      const uint8_t *src =
          Q8 ? reinterpret_cast<const uint8_t *>(v ? a.vcache : a.kcache) + (p * a.kv_heads + kvh) * RB
             : reinterpret_cast<const uint8_t *>((v ? a.vcache : a.kcache) + p * a.kv_heads * HD + kvh * HD);
      bulk_g2s(raw + ((g & 1) * CH + lane) * RB, src, (unsigned)RB, bar);
    }
  };
  bool landed = true;
  int issued = 0, waited = 0;
  for (int g = 0; g < 2 && g < 2 * nk; ++g, ++issued)
    if (warp == 0) issue(g);

  // ---- scores ----
  // warp w: leaf group w & 7, queries 8 (w >> 3) + 2 qg + x, positions pg + 8 y
  const int lg = warp & 7, q0 = 8 * (warp >> 3) + 2 * (lane >> 3), pg = lane & 7;
  float runmax = -INFINITY;
  for (int c = 0; c < nk && landed; ++c) {
    const int c0 = c * CH, cn = min(CH, plast - c0), g = c;
    landed = __syncthreads_and(mbar_wait_bounded(&bars[g & 1], (unsigned)(g >> 1) & 1u, a.status));
    if (!landed) break;
    ++waited;
    {
      const uint8_t *rb = raw + (g & 1) * CH * RB;
      const int d = tid & (HD - 1), p1 = (tid / HD) * (CH / 2);
      for (int pp = p1; pp < p1 + CH / 2; ++pp)
        rows[d * CP + pp] = pp < cn ? Ops::widen_row(rb + pp * RB, d) : Ops::widen(0.0f);
    }
    __syncthreads();
    if (g + 2 < 2 * nk) {
      if (warp == 0) {
        fence_proxy_async_smem();
        issue(g + 2);
      }
      ++issued;
    }
    // partial tree R(b, 8) = (P_b + P_b+16) + (P_b+8 + P_b+24) of leaves
    // (8-dimension chains) b = lg, for queries q0, q0+1 and positions pg+8y
    double A[2][4], B[2][4], C[2][4];
    auto leaf = [&](int l, double (&P)[2][4]) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = 8 * l + j;
        T qv[2], kv[4];
        if constexpr (Q8) {
          const float2 q2 = *reinterpret_cast<const float2 *>(qT + d * QN + q0);
          qv[0] = q2.x, qv[1] = q2.y;
        } else {
          const double2 q2 = *reinterpret_cast<const double2 *>(qT + d * QN + q0);
          qv[0] = q2.x, qv[1] = q2.y;
        }
#pragma unroll
        for (int y = 0; y < 4; y += 2) {
          // positions 2pg, 2pg+1 and 2pg+16, 2pg+17: one pair load each
          const T *kp = rows + d * CP + 2 * pg + 8 * y;
          if constexpr (Q8) {
            const float2 k2 = *reinterpret_cast<const float2 *>(kp);
            kv[y] = k2.x, kv[y + 1] = k2.y;
          } else {
            const double2 k2 = *reinterpret_cast<const double2 *>(kp);
            kv[y] = k2.x, kv[y + 1] = k2.y;
          }
        }
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y)
            P[x][y] = j == 0 ? Ops::first(qv[x], kv[y]) : Ops::next(qv[x], kv[y], P[x][y]);
      }
    };
    leaf(lg, A);
    leaf(lg + 16, B);
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) A[x][y] = A[x][y] + B[x][y];
    leaf(lg + 8, B);
    leaf(lg + 24, C);
#pragma unroll
    for (int x = 0; x < 2; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y)
        Rs[(lg * QN + q0 + x) * CH + 2 * pg + (y & 1) + 16 * (y >> 1)] =
            A[x][y] + (B[x][y] + C[x][y]);
    __syncthreads();
    // the rest of the butterfly: ((R0+R4)+(R2+R6)) + ((R1+R5)+(R3+R7)), one
    // (query, position) per thread
    {
      const int qi = tid >> 5;
      {
        const int pp = tid & 31, p = c0 + pp;
        if (pp < cn && p < qpos[qi]) {
          const double *r = Rs + qi * CH + pp;
          constexpr int st = QN * CH;
          const double s = ((r[0] + r[4 * st]) + (r[2 * st] + r[6 * st])) +
                           ((r[st] + r[5 * st]) + (r[3 * st] + r[7 * st]));
          const float sc = __fmul_rn((float)s, scale);
          S[(long)qi * pa.context + p] = sc;
          runmax = fmaxf(runmax, sc);
        }
      }
    }
    __syncthreads();  // Rs and rows are rewritten by the next chunk
  }
  // maximum of each query's scores: warp qi
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
    runmax = fmaxf(runmax, __shfl_xor_sync(0xffffffffu, runmax, off));
  if (lane == 0) {
    const int qi = warp;
    qmax[qi] = runmax;
    qM[qi] = qvalid[qi]
                 ? fmaxf(pa.scur[(long)(t0 + qi / G) * a.heads + kvh * G + qi % G], runmax)
                 : 0.0f;
  }
  __syncthreads();

  // ---- softmax ----
  // exponentials, a warp per query
  {
    const int qi = warp, pos = qpos[qi];
    const float M = qM[qi];
    float *Sq = S + (long)qi * pa.context;
#pragma unroll 8
    for (int p = lane; p < pos; p += 32) Sq[p] = exp_cr(__fsub_rn(Sq[p], M));
  }
  __syncthreads();
  // per (query, rank, warp of 32 virtual threads): the block sum's warp
  // butterfly over each virtual thread's strided binary64 total
  for (int k = tid; k < QN * 64; k += kPfThreads) {
    const int qi = k >> 6, r = (k >> 3) & 7, w = k & 7, pos = qpos[qi];
    const int per = (pos + 7) / 8, lo = min(pos, r * per), hi = min(pos, lo + per);
    const float *Sq = S + (long)qi * pa.context;
    const int base = lo + 32 * w;
    double v[32];
    if (base < hi) {
      // virtual thread l's first term (0.0 + e is e; no term leaves 0.0),
      // every load in flight at once; later terms only when per > 256
      float e0[32];
#pragma unroll
      for (int l = 0; l < 32; ++l) e0[l] = base + l < hi ? Sq[base + l] : 0.0f;
#pragma unroll
      for (int l = 0; l < 32; ++l) v[l] = (double)e0[l];
      if (base + 256 < hi) {
#pragma unroll
        for (int l = 0; l < 32; ++l)
          for (int idx = base + 256 + l; idx < hi; idx += 256) v[l] += (double)Sq[idx];
      }
      W[k] = butterfly_sum32(v);
    } else {
      W[k] = 0.0;
    }
  }
  __syncthreads();
  if (tid < QN && qvalid[tid]) {
    const int qi = tid, pos = qpos[qi], per = (pos + 7) / 8;
    double total = 0.0;
    for (int r = 0; r < 8; ++r) {
      if (min(pos, r * per) >= min(pos, min(pos, r * per) + per)) continue;  // empty rank
      double tr = 0.0;
      for (int w = 0; w < 8; ++w) tr += W[qi * 64 + r * 8 + w];
      total += tr;
    }
    const float M = qM[qi];
    const float e_cur = exp_cr(__fsub_rn(pa.scur[(long)(t0 + qi / G) * a.heads + kvh * G + qi % G], M));
    total += (double)e_cur;
    const float inv = (float)(1.0 / total);
    qinv[qi] = inv;
    qpcur[qi] = round_f16(__fmul_rn(e_cur, inv));
    if (!is_finite_f(M)) report(a.status, kStatusNonfinite);
  }
  __syncthreads();
  {
    const int qi = warp, pos = qvalid[qi] ? qpos[qi] : 0;
    const float inv = qinv[qi];
    float *Sq = S + (long)qi * pa.context;
#pragma unroll 8
    for (int p = lane; p < pos; p += 32) Sq[p] = round_f16(__fmul_rn(Sq[p], inv));
  }
  __syncthreads();

  // ---- values: thread (d, qh) = (tid % 256, tid / 256), queries 8qh.. ----
  // Each chunk is cut at the union of the queries' rank boundaries (and of
  // the ends of their position ranges); within a segment every query's
  // chain runs without a test, and at a cut the queries whose rank ends
  // there fold their partial into the rank-ordered total.
  constexpr int QH = QN / 2;
  const int d = tid & (HD - 1), qh = tid / HD, qb = QH * qh;
  // this half's QH probabilities of one position, in 16-byte loads
  auto load_probs = [](const T *src, T (&dst)[QH]) {
    if constexpr (Q8) {
#pragma unroll
      for (int x = 0; x < QH; x += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(src + x);
        dst[x] = v.x, dst[x + 1] = v.y, dst[x + 2] = v.z, dst[x + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int x = 0; x < QH; x += 2) {
        const double2 v = *reinterpret_cast<const double2 *>(src + x);
        dst[x] = v.x, dst[x + 1] = v.y;
      }
    }
  };
  double acc[QH], tot[QH];
#pragma unroll
  for (int x = 0; x < QH; ++x) {
    acc[x] = -0.0;
    tot[x] = -0.0;
  }
  // this thread's probability of the next chunk, loaded a chunk ahead
  static_assert(CH * QN == kPfThreads, "one probability per thread");
  float pnext;
  auto load_p = [&](int c0) {
    const int pp = tid / QN, qi = tid % QN, p = c0 + pp;
    pnext = p < plast && p < qpos[qi] ? S[(long)qi * pa.context + p] : 0.0f;
  };
  load_p(0);
  for (int c = 0; c < nk && landed; ++c) {
    const int c0 = c * CH, cn = min(CH, plast - c0), g = nk + c;
    landed = __syncthreads_and(mbar_wait_bounded(&bars[g & 1], (unsigned)(g >> 1) & 1u, a.status));
    if (!landed) break;
    ++waited;
    {
      const uint8_t *rb = raw + (g & 1) * CH * RB;
      const int p1 = qh * (CH / 2), p2 = min(cn, p1 + CH / 2);
      for (int pp = p1; pp < p2; ++pp) rows[pp * HD + d] = Ops::widen_row(rb + pp * RB, d);
    }
    pd[tid] = Ops::widen(pnext);
    if (tid < QN) {
      // rank boundaries of query tid inside the chunk, and its positions
      // (a query past the prompt's end runs unchecked on zero
      // probabilities; its sums are never stored)
      const int pos = qpos[tid], per = (pos + 7) / 8;
      const int cnt = qvalid[tid] ? max(0, min(cn, pos - c0)) : cn;
      unsigned m = 0;
      if (qvalid[tid] && cnt > 0) {
        int b = (c0 + per - 1) / per * per;  // first multiple of per at or after c0
        if (b == 0) b = per;
        for (; b < c0 + cnt; b += per) m |= 1u << (b - c0);
      }
      qmask[tid] = m;
      qcnt[tid] = cnt;
    }
    __syncthreads();
    if (g + 2 < 2 * nk) {
      if (warp == 0) {
        fence_proxy_async_smem();
        issue(g + 2);
      }
      ++issued;
    }
    if (c + 1 < nk) load_p(c0 + CH);
    unsigned cuts = 0;
    bool full = true;
#pragma unroll
    for (int qi = 0; qi < QN; ++qi) {
      cuts |= qmask[qi];
      if (qcnt[qi] < cn) {
        full = false;
        if (qcnt[qi] > 0) cuts |= 1u << qcnt[qi];
      }
    }
    int pp = 0;
    while (pp < cn) {
      if ((cuts >> pp) & 1u) {
#pragma unroll
        for (int x = 0; x < QH; ++x)
          if ((qmask[qb + x] >> pp) & 1u) {
            tot[x] += acc[x];
            acc[x] = -0.0;
          }
      }
      const unsigned above = pp < 31 ? cuts & ~((2u << pp) - 1u) : 0u;
      const int end = above ? min(cn, __ffs(above) - 1) : cn;
      if (full) {
        for (; pp < end; ++pp) {
          const T vv = rows[pp * HD + d];
          T pr[QH];
          load_probs(pd + pp * QN + qb, pr);
#pragma unroll
          for (int x = 0; x < QH; ++x) acc[x] = Ops::next(pr[x], vv, acc[x]);
        }
      } else {
        // the chunk where some queries' positions end: the active set is
        // constant within the segment
        bool act[QH];
#pragma unroll
        for (int x = 0; x < QH; ++x) act[x] = pp < qcnt[qb + x];
        for (; pp < end; ++pp) {
          const T vv = rows[pp * HD + d];
          T pr[QH];
          load_probs(pd + pp * QN + qb, pr);
#pragma unroll
          for (int x = 0; x < QH; ++x)
            if (act[x]) acc[x] = Ops::next(pr[x], vv, acc[x]);
        }
      }
    }
    __syncthreads();  // rows, pd and the masks are rewritten by the next chunk
  }
  // a chunk that never landed: let the copies still in flight finish
  // (bounded) before the CTA exits
  if (issued > waited && tid == 0)
    for (int g = waited; g < issued; ++g)
      mbar_wait_bounded(&bars[g & 1], (unsigned)(g >> 1) & 1u, a.status);
#pragma unroll
  for (int x = 0; x < QH; ++x) {
    const int qi = qb + x;
    if (!qvalid[qi]) continue;
    const int pos = qpos[qi], h = kvh * G + qi % G, t = t0 + qi / G;
    double sum = tot[x] + acc[x];
    const float vc =
        Q8 ? q8_0_value(reinterpret_cast<const uint8_t *>(a.vcache) + ((long)pos * a.kv_heads + kvh) * RB,
                        HD, d)
           : half_bits_to_float(a.vcache[(long)pos * a.kv_heads * HD + kvh * HD + d]);
    sum += (double)__fmul_rn(qpcur[qi], vc);
    const float out = (float)sum;
    const float gt = a.projected[(long)t * a.seq_proj + (long)(2 * h + 1) * HD + d];
    a.attended[(long)t * a.seq_out + (long)h * HD + d] = __fmul_rn(out, sigmoid_f(gt));
  }
}

__global__ void fill_positions_kernel(int *pos, int p0, int T, int *model_position) {
  for (int t = threadIdx.x; t < T; t += blockDim.x) pos[t] = p0 + t;
  if (threadIdx.x == 0 && model_position) *model_position = p0 + T;
}

}  // namespace prism

namespace prism {

// The batched attention kernel's geometry: one thread per head dimension
// (256) and whole KV groups in a CTA's kPfQueries queries.
inline bool prefill_attn_geometry(const prism_b200_qwen35_config &c) {
  const uint32_t G = c.kv_heads ? c.heads / c.kv_heads : 0;
  return c.head_dim == 256 && G >= 1 && G <= (uint32_t)kPfQueries && c.heads == G * c.kv_heads;
}

inline cudaError_t prefill_alloc(prism_b200_model *m) {
  PrefillBuffers &pb = m->pre;
  if (pb.ready) return cudaSuccess;
  const auto &c = m->cfg;
  const size_t T = kPrefillChunk;
  cudaError_t e = cudaSuccess;
  auto A = [&](auto **p, size_t count) {
    if (e == cudaSuccess) e = model_alloc(m, p, count);
  };
  A(&pb.hidden, T * c.hidden);
  A(&pb.xn, T * c.hidden);
  A(&pb.mixed, T * m->channels());
  A(&pb.zgate, T * m->value_width());
  A(&pb.beta, T * c.ssm_values);
  A(&pb.alpha, T * c.ssm_values);
  A(&pb.o_pre, T * m->value_width());
  A(&pb.act, T * m->channels());
  A(&pb.db, T * c.ssm_values * 2);
  A(&pb.attended, T * std::max<size_t>(m->value_width(), (size_t)c.heads * c.head_dim));
  A(&pb.projected, T * c.heads * c.head_dim * 2);
  A(&pb.key, T * m->kvw());
  A(&pb.value, T * m->kvw());
  A(&pb.up, T * c.ffn);
  A(&pb.gate, T * c.ffn);
  const size_t widest = std::max({(size_t)c.hidden, (size_t)c.ffn, (size_t)c.heads * c.head_dim,
                                  (size_t)m->value_width()});
  uint8_t *tok = nullptr;
  A(&tok, token_q8k_bytes(T, (int)(widest / 256)));
  pb.tok = tok;
  A(&pb.pos, T);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gdn_rows_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)gdn_scan_smem());
  if (prefill_attn_geometry(c)) {
    const size_t TQ = kPfQueries / (c.heads / c.kv_heads);
    A(&pb.qrows, T * c.heads * c.head_dim);
    A(&pb.scur, T * c.heads);
    A(&pb.scratch, (size_t)c.kv_heads * ((T + TQ - 1) / TQ) * kPfQueries * c.context);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_prefill_kernel<false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)prefill_attn_smem<false>());
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_prefill_kernel<true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)prefill_attn_smem<true>());
  }
  pb.ready = e == cudaSuccess;
  return e;
}

// Enqueue the batched pass of the T prompt tokens at positions p0 .. p0+T-1
// (already in m->d_tokens) on the model's stream; no LM head.
inline cudaError_t enqueue_prefill(prism_b200_model *m, int p0, int T) {
  PrefillBuffers &pb = m->pre;
  const auto &c = m->cfg;
  prism_b200_executor *ex = m->ex;
  cudaStream_t s = m->stream;
  unsigned *status = ex->d_status;
  const int H = (int)c.hidden, hnb = H / 256, hd = (int)c.head_dim, S = (int)c.ssm_state;
  cudaError_t e;
#define PK(x)                            \
  if ((e = (x)) != cudaSuccess) return e
  fill_positions_kernel<<<1, 256, 0, s>>>(pb.pos, p0, T, nullptr);
  PK(cudaGetLastError());
  if (c.weight_kind == 35)
    embed_batch_kernel<35><<<dim3((H + 255) / 256, T), 256, 0, s>>>(
        m->embd.units, m->embd.h, m->embd.nb, (int)c.vocab, m->d_tokens + p0, pb.hidden, H,
        status);
  else
    embed_batch_kernel<10><<<dim3((H + 255) / 256, T), 256, 0, s>>>(
        m->embd.units, m->embd.h, m->embd.nb, (int)c.vocab, m->d_tokens + p0, pb.hidden, H,
        status);
  PK(cudaGetLastError());
  auto norm = [&](const float *w) {
    rmsnorm_rows_kernel<<<T, 256, 0, s>>>(pb.hidden, w, H, c.eps, pb.xn, status);
    return cudaGetLastError();
  };
  auto quant = [&](const float *x, int nb) {
    return launch_token_quantize(x, T, nb, 0, token_q8k_carve(pb.tok, T, nb), status, s, false);
  };
  auto mm = [&](const DeviceWeight &w, float *y, const float *residual) {
    return launch_token_matmul(w, T, token_q8k_carve(pb.tok, T, w.nb), y, residual, nullptr,
                               status, s, false);
  };
  for (size_t l = 0; l < m->L.size(); ++l) {
    ModelLayer &Ly = m->L[l];
    PK(norm(Ly.attn_norm));
    PK(quant(pb.xn, hnb));
    if (Ly.full) {
      PK(mm(Ly.q, pb.projected, nullptr));
      PK(mm(Ly.k, pb.key, nullptr));
      PK(mm(Ly.v, pb.value, nullptr));
      AttnArgs aa{};
      aa.heads = (int)c.heads;
      aa.kv_heads = (int)c.kv_heads;
      aa.hd = hd;
      aa.rope_dim = (int)c.rope_dim;
      for (int j = 0; j < 3; ++j) aa.sections[j] = (int)c.rope_sections[j];
      aa.eps = c.eps;
      aa.theta_scale = powf(c.rope_base, -2.0f / (float)c.rope_dim);
      aa.projected = pb.projected;
      aa.key_in = pb.key;
      aa.value_in = pb.value;
      aa.q_norm = Ly.q_norm;
      aa.k_norm = Ly.k_norm;
      aa.kcache = Ly.kc;
      aa.vcache = Ly.vc;
      aa.q8 = c.kv_policy == PRISM_B200_KV_Q8_0 ? 1 : 0;
      aa.position = pb.pos;
      aa.pos_stride = 1;
      aa.seq_proj = (long)c.heads * hd * 2;
      aa.seq_kv_in = m->kvw();
      aa.seq_out = (long)c.heads * hd;
      aa.seq_cache = 0;  // one sequence: every token reads the same cache
      aa.no_write = 1;   // kv_rows_kernel wrote the rows
      aa.attended = pb.attended;
      aa.status = status;
      kv_rows_kernel<<<dim3(c.kv_heads, T), kAttnThreads, 0, s>>>(aa, p0);
      PK(cudaGetLastError());
      if (prefill_attn_geometry(c)) {
        const int G = (int)(c.heads / c.kv_heads), TQ = kPfQueries / G;
        query_rows_kernel<<<dim3(c.heads, T), kAttnThreads, 0, s>>>(aa, p0, pb.qrows, pb.scur);
        PK(cudaGetLastError());
        PrefillAttnArgs pa{aa, p0, T, G, TQ, (int)c.context, pb.qrows, pb.scur, pb.scratch};
        const dim3 grid(c.kv_heads, (T + TQ - 1) / TQ);
        if (aa.q8)
          attention_prefill_kernel<true><<<grid, kPfThreads, prefill_attn_smem<true>(), s>>>(pa);
        else
          attention_prefill_kernel<false><<<grid, kPfThreads, prefill_attn_smem<false>(), s>>>(pa);
        PK(cudaGetLastError());
      } else {
        // other geometries: attention_decode_kernel, one grid row per token
        const size_t smem = attn_launch_smem(aa, (int)c.context);
        cudaLaunchAttribute cattr[2];
        cudaLaunchConfig_t cfg =
            pdl_config(dim3(c.heads * kAttnSplit, T), dim3(kAttnThreads), smem, s, cattr, false);
        cattr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        cattr[cfg.numAttrs].val.clusterDim.x = kAttnSplit;
        cattr[cfg.numAttrs].val.clusterDim.y = 1;
        cattr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs += 1;
        PK(cudaLaunchKernelEx(&cfg, attention_decode_kernel, aa));
      }
      PK(quant(pb.attended, (int)(c.heads * c.head_dim / 256)));
      PK(mm(Ly.o, pb.hidden, pb.hidden));
    } else {
      PK(mm(Ly.qkv, pb.mixed, nullptr));
      PK(mm(Ly.z, pb.zgate, nullptr));
      PK(mm(Ly.beta, pb.beta, nullptr));
      PK(mm(Ly.alpha, pb.alpha, nullptr));
      const long hist_stride = (long)m->channels() * (c.conv_kernel - 1);
      const float *hist_in = Ly.conv_state + (p0 & 1) * hist_stride;
      float *hist_out = Ly.conv_state + ((p0 + T) & 1) * hist_stride;
      GdnTokensArgs g{};
      g.S = S;
      g.groups = (int)c.ssm_groups;
      g.values = (int)c.ssm_values;
      g.conv_k = (int)c.conv_kernel;
      g.T = T;
      g.channels = m->channels();
      g.eps = c.eps;
      g.mixed = pb.mixed;
      g.beta_in = pb.beta;
      g.alpha_in = pb.alpha;
      g.conv_w = Ly.conv_w;
      g.dt_bias = Ly.dt_bias;
      g.ssm_a = Ly.ssm_a;
      g.hist_in = hist_in;
      g.act = pb.act;
      g.db = pb.db;
      g.state = Ly.matrix;
      g.o_pre = pb.o_pre;
      g.status = status;
      gdn_token_inputs_kernel<<<dim3(T, 2 * c.ssm_groups + c.ssm_values), 128, 0, s>>>(g);
      PK(cudaGetLastError());
      gdn_rows_scan_kernel<<<c.ssm_values * S / kScanRows, 32 * kScanRows, gdn_scan_smem(), s>>>(g);
      PK(cudaGetLastError());
      conv_history_kernel<<<(m->channels() + 255) / 256, 256, 0, s>>>(
          pb.mixed, hist_in, hist_out, m->channels(), (int)c.conv_kernel - 1, T);
      PK(cudaGetLastError());
      gated_rows_kernel<<<T, std::min<uint32_t>(c.ssm_values, 32) * 32, 0, s>>>(pb.o_pre, pb.zgate, Ly.ssm_norm,
                                                          (int)c.ssm_values, S, c.eps,
                                                          pb.attended);
      PK(cudaGetLastError());
      PK(quant(pb.attended, m->value_width() / 256));
      PK(mm(Ly.out, pb.hidden, pb.hidden));
    }
    PK(norm(Ly.post_norm));
    PK(quant(pb.xn, hnb));
    PK(mm(Ly.up, pb.up, nullptr));
    PK(mm(Ly.gate, pb.gate, nullptr));
    {
      const long n = (long)T * c.ffn;
      swiglu_kernel<<<(unsigned)std::min<long>((n + 255) / 256, 4096), 256, 0, s>>>(
          pb.up, pb.gate, n, status);
      PK(cudaGetLastError());
    }
    PK(quant(pb.up, (int)(c.ffn / 256)));
    PK(mm(Ly.down, pb.hidden, pb.hidden));
  }
  fill_positions_kernel<<<1, 256, 0, s>>>(pb.pos, p0, T, m->d_position);
  PK(cudaGetLastError());
#undef PK
  return cudaSuccess;
}

}  // namespace prism

int prism_b200_model_prefill_async(prism_b200_model *m, size_t n) {
  using namespace prism;
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (n == 0) return ex->fail(PRISM_B200_E_INVALID, "prefill needs at least one token");
  if (m->position + (int64_t)n > (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  // rotated records: one-token steps (the reference's tiled prefill keeps
  // the sequential steps' records bit for bit, tests/graph/quantized_kv.rs:
  // 164-260)
  if (m->rotated()) return prism_b200_model_ingest_async(m, n);
  cudaSetDevice(ex->device);
  CK(prefill_alloc(m), "prefill buffers");
  for (size_t done = 0; done < n; done += kPrefillChunk) {
    const int T = (int)std::min<size_t>(kPrefillChunk, n - done);
    CK(enqueue_prefill(m, (int)(m->position + (int64_t)done), T), "prefill");
  }
  m->position += (int64_t)n;
  return PRISM_B200_OK;
}

int prism_b200_model_ingest_block(prism_b200_model *m, const uint32_t *tokens, size_t n) {
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!tokens || n == 0 || n > PRISM_B200_MAX_PREFILL_BLOCK_TOKENS)
    return ex->fail(PRISM_B200_E_INVALID, "invalid prefill block bounds");
  st = prism_b200_model_set_prompt(m, tokens, n);
  if (st) return st;
  st = prism_b200_model_prefill_async(m, n);
  if (st) return st;
  return model_finish(m);
}
