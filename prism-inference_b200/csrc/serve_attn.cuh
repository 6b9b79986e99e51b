// serve_attn.cuh -- attention of batched serving over Q8_0 KV records.
//
// One 8-CTA cluster per (sequence, KV head) computes all the query heads of
// that KV head's group (grouped-query attention reads each K and V row once
// per group, not once per query head).  CTA r takes a contiguous share of
// the cached positions and streams their K records, then their V records,
// through shared memory with bulk copies (64 positions per chunk, double
// buffered).  The cache is laid out [sequence][KV head][position] so that a
// chunk is one contiguous copy.  V rows are plain Q8_0 records (scales, then
// codes); K rows are interleaved in pages of 32 positions -- the page holds
// the scales [block][position] then the code words [word][position] -- so
// that the 32 lanes of a warp, one position each, read consecutive words.
//
// Arithmetic (the Q8_0 policy of the oracle's q8_attention, which follows
// the reference's full attention, src/graph.rs:4470-4950, Source): each
// score is float_dot(q, dequantized key) -- binary32 products summed in
// binary64 (four interleaved partial sums per thread, like the lane partials
// of the single-sequence kernel; the current position's score in dimension
// order); softmax_round_f16 with the maximum and the
// binary64 total combined over the cluster through distributed shared
// memory; values are binary64 sums of binary32 products, per CTA in
// position order and then over the CTAs in rank order; the output is gated
// by sigmoid(gate).
#pragma once

#include <cooperative_groups.h>

#include "model_kernels.cuh"

namespace prism {

constexpr int kServeSplit = 8;    // CTAs (one cluster) per (sequence, KV head)
constexpr int kServeChunk = 64;   // positions per streamed chunk
constexpr int kServeThreads = 256;
constexpr int kServeGroup = 4;    // largest query-head group
constexpr int kServePage = 32;    // positions per interleaved K page
static_assert(kServeThreads == 4 * kServeChunk, "K pass: four lanes per chunk position");

// Byte offsets, inside a K page of `hd`-dimensional rows, of position slot
// `lane`'s scale of block `blk` and its code of dimension `d`.
__host__ __device__ constexpr int kpage_scale(int hd, int blk, int lane) {
  return (blk * kServePage + lane) * 2 + 0 * hd;
}
__host__ __device__ constexpr int kpage_code(int hd, int d, int lane) {
  return kServePage * (hd / 32) * 2 + ((d >> 2) * kServePage + lane) * 4 + (d & 3);
}

struct ServeArgs {
  AttnArgs a;   // geometry, per-sequence input/output strides, norms, cache bases
  int context;  // positions per (sequence, KV head) in the cache
};

// Scores held per CTA: the largest page-aligned share of the cached
// positions, ceil(pos / (kServeSplit * kServePage)) * kServePage for
// pos < context.
__host__ __device__ constexpr int serve_cap(int context) {
  return (context + kServeSplit * kServePage - 1) / (kServeSplit * kServePage) * kServePage;
}
static_assert(serve_cap(4224) == 544 && serve_cap(8192) == 1024 && serve_cap(64) == 32,
              "serve_cap covers the page-aligned shares");

// Shared memory: q[G][hd], kc, vc, buf [hd], cs[64], scores[G][cap],
// qr[G][4][hd/4] (q regrouped by dimension residue mod 4) (f32); two chunk
// buffers; partial[G][hd] (f64); two mbarriers.
__host__ __device__ constexpr size_t serve_offset_chunks(int hd, int context) {
  return ((size_t)(2 * kServeGroup * hd + 3 * hd + 64 + kServeGroup * serve_cap(context)) * 4 +
          127) /
         128 * 128;
}
__host__ __device__ constexpr size_t serve_offset_partial(int hd, int context) {
  return serve_offset_chunks(hd, context) + 2 * (size_t)kServeChunk * q8_0_record_bytes(hd);
}
__host__ __device__ constexpr size_t serve_smem_bytes(int hd, int context) {
  return serve_offset_partial(hd, context) + (size_t)kServeGroup * hd * 8 + 16;
}

__global__ void __launch_bounds__(kServeThreads) attention_serve_kernel(ServeArgs sa) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(128) uint8_t ssm[];
  __shared__ double red[kServeThreads / 32];
  __shared__ float fred[kServeThreads / 32];
  __shared__ float s_max[kServeGroup], s_cur[kServeGroup], s_pcur[kServeGroup];
  __shared__ double s_tot[kServeGroup];
  AttnArgs a = sa.a;
  const int hd = a.hd, G = a.heads / a.kv_heads, rb = q8_0_record_bytes(hd);
  const int cap = serve_cap(sa.context);
  const int rank = (int)cluster.block_rank(), kvh = blockIdx.y;
  const long b = blockIdx.z;
  a.projected += b * a.seq_proj;
  a.key_in += b * a.seq_kv_in;
  a.value_in += b * a.seq_kv_in;
  a.attended += b * a.seq_out;
  a.position += b * a.pos_stride;
  const size_t head_bytes = (size_t)sa.context * rb;
  uint8_t *kbase = reinterpret_cast<uint8_t *>(a.kcache) + (b * a.kv_heads + kvh) * head_bytes;
  uint8_t *vbase = reinterpret_cast<uint8_t *>(a.vcache) + (b * a.kv_heads + kvh) * head_bytes;
  float *q = reinterpret_cast<float *>(ssm);  // [G][hd]
  float *kc = q + kServeGroup * hd;
  float *vc = kc + hd;
  float *buf = vc + hd;
  float *cs = buf + hd;                        // [64]
  float *scores = cs + 64;                     // [G][cap]
  float *qr = scores + kServeGroup * cap;      // [G][4][hd/4]: qr[j][e][w] = q[j][4w+e]
  uint8_t *chunks = ssm + serve_offset_chunks(hd, sa.context);
  double *partial = reinterpret_cast<double *>(ssm + serve_offset_partial(hd, sa.context));
  uint64_t *bars = reinterpret_cast<uint64_t *>(partial + kServeGroup * hd);
  const int i = threadIdx.x;
  grid_dependency_wait();
  grid_dependents_launch();
  const int pos = *a.position;
  // page-aligned shares of the cached positions
  const int per = (pos + kServeSplit * kServePage - 1) / (kServeSplit * kServePage) * kServePage;
  const int lo = min(pos, rank * per), hi = min(pos, lo + per), n = hi - lo;
  const int nchunks = (n + kServeChunk - 1) / kServeChunk;
  if (i == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init_fence();
  }
  __syncthreads();
  // chunk g of the pass sequence: K chunks 0..nchunks-1, then V chunks
  auto issue = [&](int g) {
    const bool v = g >= nchunks;
    const int c = v ? g - nchunks : g;
    int count = min(kServeChunk, n - c * kServeChunk);
    if (!v) count = (count + kServePage - 1) / kServePage * kServePage;  // whole K pages
    const uint32_t bytes = (uint32_t)(count * rb);
    uint64_t *bar = &bars[g & 1];
    mbar_arrive_expect_tx(bar, bytes);
    bulk_g2s(chunks + (g & 1) * kServeChunk * rb,
             (v ? vbase : kbase) + (size_t)(lo + c * kServeChunk) * rb, bytes, bar);
  };
  if (i == 0) {
    for (int g = 0; g < 2 && g < 2 * nchunks; ++g) issue(g);
  }
  bool ok = true;
  auto wait_chunk = [&](int g) {
    ok &= mbar_wait_bounded(&bars[g & 1], (unsigned)(g >> 1) & 1u, a.status);
  };
  // RoPE angles (reference src/graph.rs:6406-6437), the query heads of the
  // group and the current key/value of this KV head
  if (i < a.rope_dim / 2) {
    float theta = (float)pos;
    for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, a.theta_scale);
    const float angle = i < 3 * a.sections[i % 3] ? theta : 0.0f;
    cs[2 * i] = cos_cr(angle);
    cs[2 * i + 1] = sin_cr(angle);
  }
  __syncthreads();
  for (int j = 0; j < G; ++j) {
    const float qv = norm_rope_round(a.projected + (long)(kvh * G + j) * 2 * hd, a.q_norm, a.eps,
                                     hd, a.rope_dim, cs, buf, red);
    q[j * hd + i] = qv;
    qr[(j * 4 + (i & 3)) * (hd / 4) + (i >> 2)] = qv;
  }
  kc[i] = norm_rope_round(a.key_in + (long)kvh * hd, a.k_norm, a.eps, hd, a.rope_dim, cs, buf,
                          red);
  vc[i] = round_f16(a.value_in[kvh * hd + i]);
  {
    // the current K row goes to its page slot; V is a plain record
    uint16_t hb;
    int code;
    const float kq = q8_0_code(kc[i], a.status, hb, code);
    if (rank == 0) {
      uint8_t *page = kbase + (size_t)(pos / kServePage) * kServePage * rb;
      const int slot = pos % kServePage;
      if ((i & 31) == 0) *reinterpret_cast<uint16_t *>(page + kpage_scale(hd, i >> 5, slot)) = hb;
      page[kpage_code(hd, i, slot)] = (uint8_t)(int8_t)code;
    }
    kc[i] = kq;
  }
  vc[i] = q8_0_roundtrip(vc[i], rank == 0 ? vbase + (size_t)pos * rb : nullptr, hd, a.status);
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  if (i < G) {
    // the current position's score, float_dot in dimension order
    double s = -0.0;
    for (int d = 0; d < hd; ++d) s += (double)__fmul_rn(q[i * hd + d], kc[d]);
    s_cur[i] = __fmul_rn((float)s, scale);
  }
  // K pass: thread t takes position t / 4 of each chunk and dimension
  // residue e = t % 4 for every head of the group, so that each dequantized
  // key value serves all G heads; the four residues' binary64 partial sums
  // (dimensions d = 4w + e in order) meet over the four lanes of the
  // position as (s0 + s1) + (s2 + s3)
  const int nb32 = hd / 32;
  // A chunk that never lands (bounded wait) stops the passes but not the
  // cluster barriers: every CTA of the cluster reaches each cluster.sync.
  for (int c = 0; c < nchunks && ok; ++c) {
    wait_chunk(c);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const int count = min(kServeChunk, n - c * kServeChunk);
    {
      const int pp = i >> 2, e = i & 3;
      // lanes (position, residue): the 4 residues of a position share a
      // word; 8 positions per warp read consecutive words of the page
      const uint8_t *page = chunks + (c & 1) * kServeChunk * rb + (pp / kServePage) * kServePage * rb;
      const int slot = pp % kServePage;
      double s[kServeGroup];
#pragma unroll
      for (int j = 0; j < kServeGroup; ++j) s[j] = -0.0;
      for (int blk = 0; blk < nb32; ++blk) {
        const float d =
            half_bits_to_float(*reinterpret_cast<const uint16_t *>(page + kpage_scale(hd, blk, slot)));
        float k[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const uint32_t word =
              *reinterpret_cast<const uint32_t *>(page + kpage_code(hd, blk * 32 + 4 * w, slot));
          k[w] = __fmul_rn(d, (float)(int8_t)(word >> (8 * e)));
        }
#pragma unroll
        for (int j = 0; j < kServeGroup; ++j) {
          if (j < G) {
            const float4 *qe = reinterpret_cast<const float4 *>(qr + (j * 4 + e) * (hd / 4) + blk * 8);
            const float4 qa = qe[0], qb = qe[1];
            s[j] += (double)__fmul_rn(qa.x, k[0]);
            s[j] += (double)__fmul_rn(qa.y, k[1]);
            s[j] += (double)__fmul_rn(qa.z, k[2]);
            s[j] += (double)__fmul_rn(qa.w, k[3]);
            s[j] += (double)__fmul_rn(qb.x, k[4]);
            s[j] += (double)__fmul_rn(qb.y, k[5]);
            s[j] += (double)__fmul_rn(qb.z, k[6]);
            s[j] += (double)__fmul_rn(qb.w, k[7]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kServeGroup; ++j) {
        const double v1 = __shfl_down_sync(0xffffffffu, s[j], 1);
        const double v2 = __shfl_down_sync(0xffffffffu, s[j], 2);
        const double v3 = __shfl_down_sync(0xffffffffu, s[j], 3);
        if (j < G && e == 0 && pp < count)
          scores[j * cap + c * kServeChunk + pp] = __fmul_rn((float)((s[j] + v1) + (v2 + v3)), scale);
      }
    }
    __syncthreads();  // the chunk buffer is free
    if (i == 0 && c + 2 < 2 * nchunks) {
      fence_proxy_async_smem();
      issue(c + 2);
    }
  }
  // maximum over every chunk of the cluster and the current position
  for (int j = 0; j < G; ++j) {
    float m = -INFINITY;
    for (int p = i; p < n; p += kServeThreads) m = fmaxf(m, scores[j * cap + p]);
    m = block_max_f32(m, fred);
    if (i == 0) s_max[j] = m;
  }
  cluster.sync();
  float M[kServeGroup];
  for (int j = 0; j < G; ++j) {
    M[j] = s_cur[j];
    for (int r = 0; r < kServeSplit; ++r) M[j] = fmaxf(M[j], cluster.map_shared_rank(s_max, r)[j]);
  }
  for (int j = 0; j < G; ++j) {
    double tot = 0.0;
    for (int p = i; p < n; p += kServeThreads) {
      const float e = exp_cr(__fsub_rn(scores[j * cap + p], M[j]));
      scores[j * cap + p] = e;
      tot += (double)e;
    }
    tot = block_sum_f64(tot, red);
    if (i == 0) s_tot[j] = tot;
  }
  cluster.sync();
  for (int j = 0; j < G; ++j) {
    double total = 0.0;
    for (int r = 0; r < kServeSplit; ++r) total += cluster.map_shared_rank(s_tot, r)[j];
    const float e_cur = exp_cr(__fsub_rn(s_cur[j], M[j]));
    total += (double)e_cur;
    const float inv = (float)(1.0 / total);
    if (!is_finite_f(M[j]) && i == 0 && rank == 0) report(a.status, kStatusNonfinite);
    if (i == 0) s_pcur[j] = round_f16(__fmul_rn(e_cur, inv));
    for (int p = i; p < n; p += kServeThreads)
      scores[j * cap + p] = round_f16(__fmul_rn(scores[j * cap + p], inv));
  }
  __syncthreads();
  // V pass: thread i accumulates dimension i of every head of the group
  double acc[kServeGroup];
#pragma unroll
  for (int j = 0; j < kServeGroup; ++j) acc[j] = -0.0;
  for (int c = 0; c < nchunks && ok; ++c) {
    const int g = nchunks + c;
    wait_chunk(g);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const int count = min(kServeChunk, n - c * kServeChunk);
    const uint8_t *rec0 = chunks + (g & 1) * kServeChunk * rb;
    for (int pp = 0; pp < count; ++pp) {
      const uint8_t *rec = rec0 + pp * rb;
      const float d = half_bits_to_float(reinterpret_cast<const uint16_t *>(rec)[i >> 5]);
      const float v = __fmul_rn(d, (float)(int8_t)rec[nb32 * 2 + i]);
#pragma unroll
      for (int j = 0; j < kServeGroup; ++j)
        if (j < G) acc[j] += (double)__fmul_rn(scores[j * cap + c * kServeChunk + pp], v);
    }
    __syncthreads();
    if (i == 0 && g + 2 < 2 * nchunks) {
      fence_proxy_async_smem();
      issue(g + 2);
    }
  }
  for (int j = 0; j < G; ++j) partial[j * hd + i] = acc[j];
  cluster.sync();
  // CTA r finalises dimensions [r*hd/S, (r+1)*hd/S) of every head
  const int dims = hd / kServeSplit;
  if (i < G * dims) {
    const int j = i / dims, d = rank * dims + i % dims;
    double sum = -0.0;
    for (int r = 0; r < kServeSplit; ++r) sum += cluster.map_shared_rank(partial, r)[j * hd + d];
    const float out = (float)(sum + (double)__fmul_rn(s_pcur[j], vc[d]));
    const int h = kvh * G + j;
    const float gate = a.projected[(long)(2 * h + 1) * hd + d];
    a.attended[(long)h * hd + d] = __fmul_rn(out, sigmoid_f(gate));
  }
  if (!ok && i == 0) report(a.status, kStatusTimeout);
  cluster.sync();  // peers' shared memory stays live until every read is done
}

}  // namespace prism
