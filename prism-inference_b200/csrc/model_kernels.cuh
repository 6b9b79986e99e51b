// model_kernels.cuh -- decode-step kernels of the Qwen3.5-style hybrid model.
//
// Arithmetic follows the reference's Source contract: binary32 products,
// binary64 accumulation where the reference sums in binary64 (float_dot,
// f16_dot, RMS and L2 sums, softmax totals, value sums), separate multiply
// and add.  Parallel binary64 reductions reorder the sums; their binary32
// roundings agree with the reference's sequential sums except in rare
// boundary cases.  Transcendentals (exp, log, sin, cos, pow) are CUDA's,
// within a few ulp of the host libm the reference uses.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "matvec.cuh"

namespace prism {

// ---- small helpers ---------------------------------------------------------

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Block-wide binary64 sum (all threads call; red has >= warps doubles).
__device__ __forceinline__ double block_sum_f64(double v, double *red) {
  v = warp_sum_f64(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

__device__ __forceinline__ float block_max_f32(float v, float *red) {
  v = warp_max_f32(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, red[w]);
  return t;
}

__device__ __forceinline__ float sigmoid_f(float v) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-v)));
}

// reference src/graph.rs:6357-6384 recurrent_decay
__device__ __forceinline__ float recurrent_decay_f(float alpha, float time_bias, float a,
                                                   unsigned *status) {
  if (!is_finite_f(alpha) || !is_finite_f(time_bias) || !is_finite_f(a) || a > 0.0f) {
    report(status, kStatusNonfinite);
    return 0.0f;
  }
  if (a == 0.0f) return 1.0f;
  const float linear = __fadd_rn(alpha, time_bias);
  if (linear >= 88.0f) {
    if (!is_finite_f(linear)) return 0.0f;
    return exp_cr(__fmul_rn(linear, a));
  }
  const float softplus = linear > 20.0f ? linear : log_cr(__fadd_rn(1.0f, exp_cr(linear)));
  return exp_cr(__fmul_rn(softplus, a));
}

// ---- embedding row ---------------------------------------------------------

// Decode row `token` of a tiled TQ2_0 / Q2_K weight (the tied embedding):
// reference src/kernels/tquants.rs:258-268 / src/kernels/kquants.rs:146-160.
// Element i of a block: byte (i/128)*32 + i%32, shift 2*((i%128)/32).
template <int KIND>
__device__ __forceinline__ float decode_tiled(const uint8_t *units, int h, int nb, int row,
                                              int i) {
  const int t = row / h, r = row % h, b = i >> 8, e = i & 255;
  const uint8_t *unit = units + ((long)t * nb + b) * unit_bytes(KIND, h);
  const int byte = (e >> 7) * 32 + (e & 31), shift = 2 * ((e & 127) >> 5);
  const int c = byte >> 4, off = byte & 15;
  const int code = (unit[(c * h + r) * 16 + off] >> shift) & 3;
  if (KIND == 35) {
    const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(unit + 64 * h)[r]);
    return __fmul_rn((float)(code - 1), d);
  }
  const uint8_t sc = unit[64 * h + r * 16 + (e >> 4)];
  const uint16_t *dd = reinterpret_cast<const uint16_t *>(unit + 80 * h);
  const float d = half_bits_to_float(dd[r]), dmin = half_bits_to_float(dd[h + r]);
  const float t1 = __fmul_rn(__fmul_rn(d, (float)(sc & 15)), (float)code);
  return __fsub_rn(t1, __fmul_rn(dmin, (float)(sc >> 4)));
}

struct StepState {
  int *position;                 // tokens processed so far
  uint32_t *tokens;              // [context + 1] token per position
  int *prompt_end;               // first position produced by greedy selection
  unsigned long long *argmax;    // greedy key of the current step
};

template <int KIND>
__global__ void embed_kernel(const uint8_t *units, int h, int nb, int vocab, StepState st,
                             float *hidden, int n, unsigned *status) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int pos = *st.position;
  const uint32_t token = st.tokens[pos];
  if (blockIdx.x == 0 && threadIdx.x == 0) *st.argmax = 0ull;
  if (token >= (uint32_t)vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(status, kStatusInvalid);
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    hidden[i] = decode_tiled<KIND>(units, h, nb, (int)token, i);
}

// Advance the position; past the prompt, the greedy token becomes the next
// input (reference src/runtime.rs:1944-2031 generate loop, greedy selection).
__global__ void finish_step_kernel(StepState st, int write_greedy) {
  grid_dependency_wait();
  if (threadIdx.x != 0) return;
  const int pos = *st.position + 1;
  if (write_greedy && pos >= *st.prompt_end) {
    const unsigned long long key = *st.argmax;
    st.tokens[pos] = 0xffffffffu - (unsigned)(key & 0xffffffffull);
  }
  *st.position = pos;
}

// ---- Gated DeltaNet decode step ------------------------------------------

struct GdnArgs {
  int S;             // state size (key dim = value dim per head)
  int groups;        // key heads
  int values;        // value heads
  int conv_k;        // convolution kernel (history = conv_k - 1)
  float eps;
  // per-sequence inputs (batch stride in elements)
  const float *mixed;      // [conv channels] qkv projection, before conv
  const float *zgate;      // [values*S]
  const float *beta_in;    // [values]
  const float *alpha_in;   // [values]
  long in_stride, z_stride, ab_stride;
  const float *conv_w;     // [channels][conv_k]
  const float *dt_bias, *ssm_a, *norm_w;
  float *conv_state;       // two buffers of [batch][channels][conv_k-1], by position parity
  long conv_buf_stride;    // elements between the two buffers
  long conv_stride;        // per sequence
  float *state;            // [batch][values][S][S], updated in place
  long state_stride;
  float *attended;         // [batch][values*S]
  long out_stride;
  const int *position;     // selects the conv-state buffer (nullptr: buffer 0 -> 1)
  unsigned *status;
  unsigned long long *trace;  // optional timeline, as MvArgs::trace ([0], [1], [6], [7])
};

// One CTA per (value head, sequence); 512 threads; S == 128.
// reference src/graph.rs:5029-5181 (conv, SiLU, L2 of q/k) and
// src/graph.rs:5191-5343 with gdn_step_row_from (src/graph.rs:801-822).
constexpr int kGdnThreads = 512;

__global__ void __launch_bounds__(kGdnThreads) gdn_decode_kernel(GdnArgs a) {
  constexpr int S = 128;
  __shared__ __align__(16) float q[S], k[S], v[S], o[S];
  __shared__ double red[kGdnThreads / 32];
  __shared__ float sdecay, sbeta;
  const int h = blockIdx.x, b = blockIdx.y;
  const int kh = h % a.groups;
  const int kw = a.groups * S;
  const int hist = a.conv_k - 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The state rows were written by this layer's previous step, not by the
  // kernels this one depends on: load them before the grid dependency, so
  // their HBM latency overlaps the producer's tail.
  float *state = a.state + b * a.state_stride + (long)h * S * S;
  constexpr int RPW = S / (kGdnThreads / 32);  // rows per warp (8)
  float4 srow[RPW];
  trace_stamp(a.trace, 0);
#pragma unroll
  for (int i = 0; i < RPW; ++i)
    srow[i] = reinterpret_cast<const float4 *>(state + (long)(warp * RPW + i) * S)[lane];
  grid_dependency_wait();
  trace_stamp(a.trace, 1);
  grid_dependents_launch();
  const float *mixed = a.mixed + b * a.in_stride;
  const int parity = a.position ? (*a.position & 1) : 0;
  const float *hist_in = a.conv_state + parity * a.conv_buf_stride + b * a.conv_stride;
  float *hist_out = a.conv_state + (parity ^ 1) * a.conv_buf_stride + b * a.conv_stride;

  // 1. depthwise causal convolution + SiLU of this head's q, k, v channels
  if (threadIdx.x < 3 * S) {
    const int part = threadIdx.x / S, j = threadIdx.x % S;
    const int ch = part == 0 ? kh * S + j : part == 1 ? kw + kh * S + j : 2 * kw + h * S + j;
    const float projected = mixed[ch];
    const float *hj = hist_in + (long)ch * hist;
    const float *cj = a.conv_w + (long)ch * a.conv_k;
    float sum = 0.0f;
    for (int i = 0; i < hist; ++i) sum = __fadd_rn(sum, __fmul_rn(hj[i], cj[i]));
    sum = __fadd_rn(sum, __fmul_rn(projected, cj[hist]));
    const float act = silu_f(sum);
    (part == 0 ? q : part == 1 ? k : v)[j] = act;
    // the history of shared q/k channels is written by their first value head
    if (part == 2 || h == kh) {
      float *nj = hist_out + (long)ch * hist;
      for (int i = 0; i + 1 < hist; ++i) nj[i] = hj[i + 1];
      if (hist > 0) nj[hist - 1] = projected;
    }
  }
  if (threadIdx.x == 0) {
    sdecay = recurrent_decay_f(a.alpha_in[b * a.ab_stride + h], a.dt_bias[h], a.ssm_a[h],
                               a.status);
    sbeta = sigmoid_f(a.beta_in[b * a.ab_stride + h]);
  }
  __syncthreads();
  // 2. L2 normalisation of q and k (reference src/kernels.rs:3333-3352)
  {
    const float xq = threadIdx.x < S ? q[threadIdx.x] : 0.0f;
    const float xk = threadIdx.x < S ? k[threadIdx.x] : 0.0f;
    const double sq = block_sum_f64(threadIdx.x < S ? (double)__fmul_rn(xq, xq) : 0.0, red);
    const double sk = block_sum_f64(threadIdx.x < S ? (double)__fmul_rn(xk, xk) : 0.0, red);
    const float scq = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sq), a.eps));
    const float sck = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sk), a.eps));
    __syncthreads();
    if (threadIdx.x < S) {
      q[threadIdx.x] = __fmul_rn(xq, scq);
      k[threadIdx.x] = __fmul_rn(xk, sck);
    }
  }
  __syncthreads();
  // 3. state rows: S = decay*prev; dk = S.k; delta = (v-dk)*beta;
  //    S += delta*k; o = (S.q)/sqrt(S)
  const float decay = sdecay, beta = sbeta;
  const float oscale = __fdiv_rn(1.0f, __fsqrt_rn((float)S));
  const float4 kk = reinterpret_cast<const float4 *>(k)[lane];
  const float4 qq = reinterpret_cast<const float4 *>(q)[lane];
  bool finite = true;
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int r = warp * RPW + i;
    float4 s = srow[i];
    s.x = __fmul_rn(decay, s.x);
    s.y = __fmul_rn(decay, s.y);
    s.z = __fmul_rn(decay, s.z);
    s.w = __fmul_rn(decay, s.w);
    double dk = (double)__fmul_rn(s.x, kk.x) + (double)__fmul_rn(s.y, kk.y) +
                (double)__fmul_rn(s.z, kk.z) + (double)__fmul_rn(s.w, kk.w);
    dk = warp_sum_f64(dk);
    const float delta = __fmul_rn(__fsub_rn(v[r], (float)dk), beta);
    s.x = __fadd_rn(s.x, __fmul_rn(delta, kk.x));
    s.y = __fadd_rn(s.y, __fmul_rn(delta, kk.y));
    s.z = __fadd_rn(s.z, __fmul_rn(delta, kk.z));
    s.w = __fadd_rn(s.w, __fmul_rn(delta, kk.w));
    finite &= is_finite_f(s.x) && is_finite_f(s.y) && is_finite_f(s.z) && is_finite_f(s.w);
    double dq = (double)__fmul_rn(s.x, qq.x) + (double)__fmul_rn(s.y, qq.y) +
                (double)__fmul_rn(s.z, qq.z) + (double)__fmul_rn(s.w, qq.w);
    dq = warp_sum_f64(dq);
    reinterpret_cast<float4 *>(state + (long)r * S)[lane] = s;
    if (lane == 0) o[r] = __fmul_rn((float)dq, oscale);
  }
  if (!__all_sync(0xffffffffu, finite) && lane == 0) report(a.status, kStatusNonfinite);
  __syncthreads();
  // 4. RMSNorm(o) * w * SiLU(z) (reference src/kernels.rs:3589-3625, Source)
  const float ov = threadIdx.x < S ? o[threadIdx.x] : 0.0f;
  const double ss = block_sum_f64(threadIdx.x < S ? (double)__fmul_rn(ov, ov) : 0.0, red);
  const float mean = (float)(ss / (double)S);
  const float nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
  if (threadIdx.x < S) {
    const float z = a.zgate[b * a.z_stride + h * S + threadIdx.x];
    const float normed = __fmul_rn(__fmul_rn(ov, nscale), a.norm_w[threadIdx.x]);
    a.attended[b * a.out_stride + h * S + threadIdx.x] = __fmul_rn(normed, silu_f(z));
  }
  trace_exit(a.trace);
}

// ---- gated full attention over a binary16 KV cache -------------------------

struct AttnArgs {
  int heads, kv_heads, hd, rope_dim;
  int sections[3];          // mRoPE sections (text positions: t, h, w equal)
  float eps, theta_scale;
  const float *projected;   // [heads][2][hd]: query then gate per head
  const float *key_in;      // [kv_heads*hd]
  const float *value_in;    // [kv_heads*hd]
  const float *q_norm, *k_norm;
  uint16_t *kcache, *vcache;  // [context][kv_heads*hd] binary16 bits, or Q8_0 records
  int q8;                     // 1: Q8_0 records [context][kv_heads][hd/32 scales | hd codes]
  // batched decode (grid y = sequence): per-sequence strides, 0 for one sequence
  long seq_proj, seq_kv_in, seq_out, seq_cache;  // elements of each array's own type
  int pos_stride;             // 1: position[sequence]; 0: one shared position
  const int *position;
  float *attended;          // [heads*hd]
  unsigned *status;
  // > 0: shared-memory offset of the staged K and V rows of a CTA's chunk
  // (attention_decode_kernel); 0: read them from global memory in place
  int kv_smem_off;
  unsigned long long *trace;  // optional timeline, as MvArgs::trace ([0], [1], [6], [7])
  int no_write;  // 1: the token's K/V rows are already in the cache (batched prefill)
};

constexpr int kAttnThreads = 256;

// RMSNorm(x)*w, RoPE on the first rope_dim dims, binary16 rounding
// (reference src/kernels.rs:3679-3750, Source).  One value per thread
// (hd == blockDim.x); cs holds the (cos, sin) pairs.
__device__ __forceinline__ float norm_rope_round(const float *x, const float *w, float eps,
                                                 int hd, int rope, const float *cs, float *buf,
                                                 double *red) {
  const int i = threadIdx.x;
  const float xi = x[i];
  const double ss = block_sum_f64((double)__fmul_rn(xi, xi), red);
  const float mean = (float)(ss / (double)hd);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  buf[i] = __fmul_rn(__fmul_rn(xi, scale), w[i]);
  __syncthreads();
  float out = buf[i];
  const int half = rope / 2;
  if (i < half) {
    const float first = buf[i], second = buf[i + half];
    out = __fsub_rn(__fmul_rn(first, cs[2 * i]), __fmul_rn(second, cs[2 * i + 1]));
  } else if (i < rope) {
    const int j = i - half;
    const float first = buf[j], second = buf[i];
    out = __fadd_rn(__fmul_rn(first, cs[2 * j + 1]), __fmul_rn(second, cs[2 * j]));
  }
  __syncthreads();
  return round_f16(out);
}

// Q8_0 record of one KV head's row (an addition of this build): thread i
// (i < hd) holds value i; each warp codes one 32-value block with the
// reference's Source Q8_0 codec (src/kernels.rs:552-617: d = max|x|/127,
// stored as binary16, codes = round-half-away(x * (1/d))).  Writes the
// record when `rec` is set and returns the dequantized value scale*code.
__device__ __forceinline__ float q8_0_code(float x, unsigned *status, uint16_t &hb, int &q) {
  float m = fabsf(x);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const float d = __fdiv_rn(m, 127.0f);
  const float inv = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
  hb = float_to_half_bits(d);
  float r = roundf(__fmul_rn(x, inv));
  if (!(r >= -127.0f && r <= 127.0f)) {
    report(status, kStatusInvalid);
    r = 0.0f;
  }
  q = (int)r;
  return __fmul_rn(half_bits_to_float(hb), (float)q);
}

__device__ __forceinline__ float q8_0_roundtrip(float x, uint8_t *rec, int hd,
                                                unsigned *status) {
  const int i = threadIdx.x;
  uint16_t hb;
  int q;
  const float v = q8_0_code(x, status, hb, q);
  if (rec) {
    if ((i & 31) == 0) reinterpret_cast<uint16_t *>(rec)[i >> 5] = hb;
    rec[hd / 32 * 2 + i] = (uint8_t)(int8_t)q;
  }
  return v;
}

__host__ __device__ constexpr int q8_0_record_bytes(int hd) { return hd / 32 * 2 + hd; }

// Dequantized value j of a Q8_0 record.
__device__ __forceinline__ float q8_0_value(const uint8_t *rec, int hd, int j) {
  const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(rec)[j >> 5]);
  return __fmul_rn(d, (float)(int8_t)rec[hd / 32 * 2 + j]);
}

// Score of position p: lane holds q dims lane*8..lane*8+7; binary32 products
// summed in binary64 (the binary16 or the Q8_0 key row).
__device__ __forceinline__ double key_partial(const AttnArgs &a, int p, int kvh,
                                              const float4 &q0, const float4 &q1, int lane) {
  const int hd = a.hd;
  float k[8];
  if (a.q8) {
    const int rb = q8_0_record_bytes(hd);
    const uint8_t *rec = reinterpret_cast<const uint8_t *>(a.kcache) +
                         ((long)p * a.kv_heads + kvh) * rb;
    const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(rec)[lane >> 2]);
    const uint2 c = *reinterpret_cast<const uint2 *>(rec + hd / 32 * 2 + lane * 8);
    const int8_t *cb = reinterpret_cast<const int8_t *>(&c);
#pragma unroll
    for (int j = 0; j < 8; ++j) k[j] = __fmul_rn(d, (float)cb[j]);
  } else {
    const uint4 kv = *reinterpret_cast<const uint4 *>(a.kcache + (long)p * a.kv_heads * hd +
                                                      kvh * hd + lane * 8);
    const uint16_t *kh = reinterpret_cast<const uint16_t *>(&kv);
#pragma unroll
    for (int j = 0; j < 8; ++j) k[j] = half_bits_to_float(kh[j]);
  }
  return (double)__fmul_rn(q0.x, k[0]) + (double)__fmul_rn(q0.y, k[1]) +
         (double)__fmul_rn(q0.z, k[2]) + (double)__fmul_rn(q0.w, k[3]) +
         (double)__fmul_rn(q1.x, k[4]) + (double)__fmul_rn(q1.y, k[5]) +
         (double)__fmul_rn(q1.z, k[6]) + (double)__fmul_rn(q1.w, k[7]);
}

// Value dimension i of position p (binary16 or Q8_0 row).
__device__ __forceinline__ float value_at(const AttnArgs &a, int p, int kvh, int i) {
  if (a.q8) {
    const int rb = q8_0_record_bytes(a.hd);
    return q8_0_value(reinterpret_cast<const uint8_t *>(a.vcache) +
                          ((long)p * a.kv_heads + kvh) * rb,
                      a.hd, i);
  }
  return half_bits_to_float(a.vcache[(long)p * a.kv_heads * a.hd + kvh * a.hd + i]);
}

// Attention decode for one query head split over a cluster of kAttnSplit
// CTAs (one per SM): CTA r scores and accumulates its contiguous share of
// the cached positions; the softmax maximum, the binary64 total and the
// binary64 value partial sums are combined through distributed shared
// memory in rank (= position) order.  hd == 256 == blockDim.x.
//
// Arithmetic (reference src/graph.rs:4470-4950, Source): q and the current
// k are RMS-normed, RoPE'd and rounded to binary16; past scores are f16_dot
// (binary32 products, binary64 sum) x 1/sqrt(hd), the current score a
// float_dot; softmax_round_f16 (binary64 total, probabilities rounded to
// binary16); values are binary64 sums of binary32 products, rounded once;
// the output is gated by sigmoid(gate).
constexpr int kAttnSplit = 8;

__host__ __device__ constexpr int attn_chunk_cap(int context) {
  return (context + kAttnSplit - 1) / kAttnSplit + 1;
}

__host__ __device__ constexpr size_t attn_smem_bytes(int hd, int context) {
  return ((size_t)(4 * hd + 64 + attn_chunk_cap(context)) * 4 + 15) / 16 * 16 +
         (size_t)hd * 8;
}

// Bytes of one cached position of one KV head (binary16 row or Q8_0 record).
__host__ __device__ constexpr int attn_row_bytes(int hd, int q8) {
  return q8 ? q8_0_record_bytes(hd) : hd * 2;
}

// K and V rows stream through two shared-memory buffers of kAttnChunk
// positions (placed after the layout above): K chunks for the scores, then
// V chunks for the values.
constexpr int kAttnChunk = 32;
__host__ __device__ constexpr size_t attn_smem_bytes_staged(int hd, int context, int q8) {
  return attn_smem_bytes(hd, context) + 2 * (size_t)kAttnChunk * (size_t)attn_row_bytes(hd, q8);
}

// Score of position p from a staged row (lane holds q dims lane*8..+7).
__device__ __forceinline__ double key_partial_staged(const uint8_t *row, int hd, int q8,
                                                     const float4 &q0, const float4 &q1,
                                                     int lane) {
  float k[8];
  if (q8) {
    const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(row)[lane >> 2]);
    const uint2 c = *reinterpret_cast<const uint2 *>(row + hd / 32 * 2 + lane * 8);
    const int8_t *cb = reinterpret_cast<const int8_t *>(&c);
#pragma unroll
    for (int j = 0; j < 8; ++j) k[j] = __fmul_rn(d, (float)cb[j]);
  } else {
    const uint4 kv = reinterpret_cast<const uint4 *>(row)[lane];
    const uint16_t *kh = reinterpret_cast<const uint16_t *>(&kv);
#pragma unroll
    for (int j = 0; j < 8; ++j) k[j] = half_bits_to_float(kh[j]);
  }
  return (double)__fmul_rn(q0.x, k[0]) + (double)__fmul_rn(q0.y, k[1]) +
         (double)__fmul_rn(q0.z, k[2]) + (double)__fmul_rn(q0.w, k[3]) +
         (double)__fmul_rn(q1.x, k[4]) + (double)__fmul_rn(q1.y, k[5]) +
         (double)__fmul_rn(q1.z, k[6]) + (double)__fmul_rn(q1.w, k[7]);
}

__device__ __forceinline__ float value_staged(const uint8_t *row, int hd, int q8, int i) {
  if (q8) return q8_0_value(row, hd, i);
  return half_bits_to_float(reinterpret_cast<const uint16_t *>(row)[i]);
}

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(AttnArgs args) {
  namespace cg = cooperative_groups;
  AttnArgs a = args;
  {
    const long b = blockIdx.y;  // sequence of a batched step
    a.projected += b * a.seq_proj;
    a.key_in += b * a.seq_kv_in;
    a.value_in += b * a.seq_kv_in;
    a.attended += b * a.seq_out;
    a.kcache += b * a.seq_cache;
    a.vcache += b * a.seq_cache;
    a.position += b * a.pos_stride;
  }
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float sm[];
  const int hd = a.hd;
  float *q = sm;                 // [hd]
  float *kc = q + hd;            // [hd]
  float *vc = kc + hd;           // [hd]
  float *buf = vc + hd;          // [hd]
  float *cs = buf + hd;          // [64]: (cos, sin) pairs
  float *scores = cs + 64;       // [chunk]
  double *partial;               // [hd], after the chunk's scores
  __shared__ double red[kAttnThreads / 32];
  __shared__ float fred[kAttnThreads / 32];
  __shared__ float s_max, s_cur;
  __shared__ double s_tot;
  __shared__ __align__(8) uint64_t kvbar[2];
  const int rank = (int)cluster.block_rank();
  const int h = blockIdx.x / kAttnSplit;
  const int group = a.heads / a.kv_heads;
  const int kvh = h / group;
  const int kvw = a.kv_heads * hd;
  const int i = threadIdx.x;
  const int warp = i >> 5, lane = i & 31;
  trace_stamp(a.trace, 0);
  // The position and the cached rows before it were written by earlier
  // steps, not by the kernels this one depends on: read the position, build
  // the RoPE table and start staging this CTA's K and V rows before the grid
  // dependency, so their latency overlaps the producer's tail.
  const int pos = *a.position;
  // chunk of past positions owned by this CTA
  const int per = (pos + kAttnSplit - 1) / kAttnSplit;
  const int lo = min(pos, rank * per), hi = min(pos, lo + per);
  partial = reinterpret_cast<double *>(reinterpret_cast<uint8_t *>(sm) +
                                       ((size_t)(4 * hd + 64 + per + 1) * 4 + 15) / 16 * 16);
  const bool staged = a.kv_smem_off > 0;
  const int rb = attn_row_bytes(hd, a.q8);
  uint8_t *kvbuf = reinterpret_cast<uint8_t *>(sm) + a.kv_smem_off;  // [2][kAttnChunk][rb]
  const int nk = (hi - lo + kAttnChunk - 1) / kAttnChunk;  // chunks per pass
  // chunk g of the pass sequence: K chunks 0..nk-1, then V chunks; warp 0
  // issues one bulk copy per row (lane = row) into buffer g & 1
  auto issue = [&](int g) {
    const bool v = g >= nk;
    const int p0 = lo + (v ? g - nk : g) * kAttnChunk, count = min(kAttnChunk, hi - p0);
    uint64_t *bar = &kvbar[g & 1];
    if (lane == 0) mbar_arrive_expect_tx(bar, (unsigned)(count * rb));
    __syncwarp();
    if (lane < count) {
      const int p = p0 + lane;
      const size_t at = a.q8 ? ((size_t)p * a.kv_heads + kvh) * rb
                             : ((size_t)p * kvw + (size_t)kvh * hd) * 2;
      bulk_g2s(kvbuf + ((size_t)(g & 1) * kAttnChunk + lane) * rb,
               reinterpret_cast<const uint8_t *>(v ? a.vcache : a.kcache) + at, (unsigned)rb,
               bar);
    }
  };
  bool landed = true;
  int issued = 0, waited = 0;  // chunks, identical in every thread
  if (staged) {
    if (i == 0) {
      mbar_init(&kvbar[0], 1);
      mbar_init(&kvbar[1], 1);
      mbar_init_fence();
    }
    __syncthreads();
    for (int g = 0; g < 2 && g < 2 * nk; ++g, ++issued)
      if (warp == 0) issue(g);
  }
  if (i < a.rope_dim / 2) {
    // reference src/graph.rs:6406-6437: angle_j = p * theta_scale^j by j
    // repeated binary32 multiplications; text positions give the three
    // sections the same angle, and indices past 3*section use position 0
    float theta = (float)pos;
    for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, a.theta_scale);
    const float angle = i < 3 * a.sections[i % 3] ? theta : 0.0f;
    cs[2 * i] = cos_cr(angle);
    cs[2 * i + 1] = sin_cr(angle);
  }
  grid_dependency_wait();
  trace_stamp(a.trace, 1);
  grid_dependents_launch();
  __syncthreads();
  q[i] = norm_rope_round(a.projected + (long)h * 2 * hd, a.q_norm, a.eps, hd, a.rope_dim, cs,
                         buf, red);
  kc[i] = norm_rope_round(a.key_in + (long)kvh * hd, a.k_norm, a.eps, hd, a.rope_dim, cs, buf,
                          red);
  vc[i] = round_f16(a.value_in[kvh * hd + i]);
  const bool writer = rank == 0 && h % group == 0 && !a.no_write;
  if (a.q8) {
    const int rb = q8_0_record_bytes(hd);
    const long at = ((long)pos * a.kv_heads + kvh) * rb;
    kc[i] = q8_0_roundtrip(kc[i], writer ? reinterpret_cast<uint8_t *>(a.kcache) + at : nullptr,
                           hd, a.status);
    vc[i] = q8_0_roundtrip(vc[i], writer ? reinterpret_cast<uint8_t *>(a.vcache) + at : nullptr,
                           hd, a.status);
  } else if (writer) {
    a.kcache[(long)pos * kvw + kvh * hd + i] = float_to_half_bits(kc[i]);
    a.vcache[(long)pos * kvw + kvh * hd + i] = float_to_half_bits(vc[i]);
  }
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  // scores of this chunk: warp per position, lane owns 8 dims (16-byte load)
  const float4 q0 = reinterpret_cast<const float4 *>(q)[lane * 2];
  const float4 q1 = reinterpret_cast<const float4 *>(q)[lane * 2 + 1];
  if (staged) {
    for (int c = 0; c < nk && landed; ++c) {
      landed = __syncthreads_and(mbar_wait_bounded(&kvbar[c & 1], (unsigned)(c >> 1) & 1u,
                                                   a.status));
      if (!landed) break;
      ++waited;
      const int p0 = lo + c * kAttnChunk, count = min(kAttnChunk, hi - p0);
      const uint8_t *rows = kvbuf + (size_t)(c & 1) * kAttnChunk * rb;
      for (int pp = warp; pp < count; pp += kAttnThreads / 32) {
        const double s =
            warp_sum_f64(key_partial_staged(rows + (size_t)pp * rb, hd, a.q8, q0, q1, lane));
        if (lane == 0) scores[p0 + pp - lo] = __fmul_rn((float)s, scale);
      }
      __syncthreads();  // the buffer is free again
      if (c + 2 < 2 * nk) {
        if (warp == 0) {
          fence_proxy_async_smem();
          issue(c + 2);
        }
        ++issued;
      }
    }
  } else {
    for (int p = lo + warp; p < hi; p += kAttnThreads / 32) {
      const double s = warp_sum_f64(key_partial(a, p, kvh, q0, q1, lane));
      if (lane == 0) scores[p - lo] = __fmul_rn((float)s, scale);
    }
  }
  {
    // the current position's score (every CTA computes the same value)
    const double s = block_sum_f64((double)__fmul_rn(q[i], kc[i]), red);
    if (i == 0) s_cur = __fmul_rn((float)s, scale);
  }
  __syncthreads();
  float m = -INFINITY;
  for (int p = i; p < hi - lo; p += kAttnThreads) m = fmaxf(m, scores[p]);
  m = block_max_f32(m, fred);
  if (i == 0) s_max = m;
  cluster.sync();
  // global maximum over every chunk and the current position
  float M = s_cur;
  for (int r = 0; r < kAttnSplit; ++r) M = fmaxf(M, *cluster.map_shared_rank(&s_max, r));
  double tot = 0.0;
  for (int p = i; p < hi - lo; p += kAttnThreads) {
    const float e = exp_cr(__fsub_rn(scores[p], M));
    scores[p] = e;
    tot += (double)e;
  }
  tot = block_sum_f64(tot, red);
  if (i == 0) s_tot = tot;
  cluster.sync();
  double total = 0.0;
  for (int r = 0; r < kAttnSplit; ++r) total += *cluster.map_shared_rank(&s_tot, r);
  const float e_cur = exp_cr(__fsub_rn(s_cur, M));
  total += (double)e_cur;
  const float inv = (float)(1.0 / total);
  if (!is_finite_f(M) && i == 0 && rank == 0) report(a.status, kStatusNonfinite);
  const float p_cur = round_f16(__fmul_rn(e_cur, inv));
  for (int p = i; p < hi - lo; p += kAttnThreads) scores[p] = round_f16(__fmul_rn(scores[p], inv));
  __syncthreads();
  // value partial sums of this chunk: one dimension per thread, position order
  if (staged) {
    double acc = -0.0;
    for (int c = 0; c < nk && landed; ++c) {
      const int g = nk + c;
      landed = __syncthreads_and(mbar_wait_bounded(&kvbar[g & 1], (unsigned)(g >> 1) & 1u,
                                                   a.status));
      if (!landed) break;
      ++waited;
      const int p0 = lo + c * kAttnChunk, count = min(kAttnChunk, hi - p0);
      const uint8_t *rows = kvbuf + (size_t)(g & 1) * kAttnChunk * rb;
      for (int pp = 0; pp < count; ++pp)
        acc += (double)__fmul_rn(scores[p0 + pp - lo],
                                 value_staged(rows + (size_t)pp * rb, hd, a.q8, i));
      __syncthreads();
      if (g + 2 < 2 * nk) {
        if (warp == 0) {
          fence_proxy_async_smem();
          issue(g + 2);
        }
        ++issued;
      }
    }
    partial[i] = acc;
    // a chunk that never landed: let the copies still in flight finish
    // (bounded) before the CTA exits
    if (issued > waited && i == 0)
      for (int g = waited; g < issued; ++g)
        mbar_wait_bounded(&kvbar[g & 1], (unsigned)(g >> 1) & 1u, a.status);
  } else {
    double acc = -0.0;
    int p = lo;
    for (; p + 4 <= hi; p += 4) {
      const float v0 = value_at(a, p, kvh, i), v1 = value_at(a, p + 1, kvh, i);
      const float v2 = value_at(a, p + 2, kvh, i), v3 = value_at(a, p + 3, kvh, i);
      acc += (double)__fmul_rn(scores[p - lo], v0);
      acc += (double)__fmul_rn(scores[p + 1 - lo], v1);
      acc += (double)__fmul_rn(scores[p + 2 - lo], v2);
      acc += (double)__fmul_rn(scores[p + 3 - lo], v3);
    }
    for (; p < hi; ++p) acc += (double)__fmul_rn(scores[p - lo], value_at(a, p, kvh, i));
    partial[i] = acc;
  }
  cluster.sync();
  // CTA r finalises dimensions [r*hd/S, (r+1)*hd/S)
  const int dims = hd / kAttnSplit;
  if (i < dims) {
    const int d = rank * dims + i;
    double sum = -0.0;
    for (int r = 0; r < kAttnSplit; ++r) sum += cluster.map_shared_rank(partial, r)[d];
    const float out = (float)(sum + (double)__fmul_rn(p_cur, vc[d]));
    const float g = a.projected[(long)(2 * h + 1) * hd + d];
    a.attended[(long)h * hd + d] = __fmul_rn(out, sigmoid_f(g));
  }
  cluster.sync();  // peers' shared memory stays live until every read is done
  trace_exit(a.trace);
}

}  // namespace prism
