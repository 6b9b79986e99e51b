// gdn.cuh -- Gated DeltaNet recurrence kernels (decode step and chunked
// prefill) for batches of sequences.
//
// Per value head h (key head h % key_heads), state rows r (value channels):
//   S_r <- decay * S_r;  delta_r = (v_r - S_r.k) * beta;  S_r += delta_r k;
//   o_r = (S_r . q) / sqrt(d)
// (reference src/graph.rs:801-822 gdn_step_row_from and 5191-5343; batched
// form of src/backend/gdn.rs:24-300 with the gate given as the decay).
//
// Layouts (f32, device):  state [batch][heads][d][d] (row r = value channel)
//   q, k [batch][T][key_heads][d];  v, out [batch][T][heads][d];
//   decay, beta [batch][T][heads].  Decode is T = 1.
#pragma once

#include "common.cuh"

namespace prism {

struct GdnBatchArgs {
  int batch, T, heads, key_heads;
  float *state;
  const float *q, *k, *v, *decay, *beta;
  float *out;
  unsigned *status;
};

__device__ __forceinline__ double gdn_warp_sum(double v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// ---- decode: one recurrent step ------------------------------------------
// grid (split, heads, batch); each CTA owns 128/split consecutive state rows
// of one (sequence, head); a warp updates one row at a time with binary32
// products summed in binary64 (the reference's float_dot), unfused updates.
constexpr int kGdnStepThreads = 256;
constexpr int kGdnRowBatch = 4;  // state rows a warp loads at once

__global__ void __launch_bounds__(kGdnStepThreads) gdn_step_kernel(GdnBatchArgs a) {
  constexpr int D = 128;
  const int split = gridDim.x;
  const int rows = D / split;
  const int r0 = blockIdx.x * rows;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h % a.key_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_dependency_wait();
  grid_dependents_launch();
  const long qk = ((long)b * a.key_heads + kh) * D;
  const long hv = ((long)b * a.heads + h) * D;
  const float4 kk = reinterpret_cast<const float4 *>(a.k + qk)[lane];
  const float4 qq = reinterpret_cast<const float4 *>(a.q + qk)[lane];
  const float decay = a.decay[(long)b * a.heads + h];
  const float beta = a.beta[(long)b * a.heads + h];
  const float oscale = __fdiv_rn(1.0f, __fsqrt_rn((float)D));
  float *state = a.state + ((long)b * a.heads + h) * D * D;
  bool finite = true;
  // a warp's rows r = r0 + warp + 8i: up to kGdnRowBatch of them are loaded
  // together, so their HBM latencies overlap
  constexpr int W = kGdnStepThreads / 32;
  for (int rb = r0 + warp; rb < r0 + rows; rb += W * kGdnRowBatch) {
    float4 sr[kGdnRowBatch];
#pragma unroll
    for (int i = 0; i < kGdnRowBatch; ++i)
      if (rb + W * i < r0 + rows)
        sr[i] = reinterpret_cast<const float4 *>(state + (long)(rb + W * i) * D)[lane];
#pragma unroll
    for (int i = 0; i < kGdnRowBatch; ++i) {
    const int r = rb + W * i;
    if (r >= r0 + rows) break;
    float4 s = sr[i];
    s.x = __fmul_rn(decay, s.x);
    s.y = __fmul_rn(decay, s.y);
    s.z = __fmul_rn(decay, s.z);
    s.w = __fmul_rn(decay, s.w);
    double dk = (double)__fmul_rn(s.x, kk.x) + (double)__fmul_rn(s.y, kk.y) +
                (double)__fmul_rn(s.z, kk.z) + (double)__fmul_rn(s.w, kk.w);
    dk = gdn_warp_sum(dk);
    const float delta = __fmul_rn(__fsub_rn(a.v[hv + r], (float)dk), beta);
    s.x = __fadd_rn(s.x, __fmul_rn(delta, kk.x));
    s.y = __fadd_rn(s.y, __fmul_rn(delta, kk.y));
    s.z = __fadd_rn(s.z, __fmul_rn(delta, kk.z));
    s.w = __fadd_rn(s.w, __fmul_rn(delta, kk.w));
    finite &= is_finite_f(s.x) && is_finite_f(s.y) && is_finite_f(s.z) && is_finite_f(s.w);
    double dq = (double)__fmul_rn(s.x, qq.x) + (double)__fmul_rn(s.y, qq.y) +
                (double)__fmul_rn(s.z, qq.z) + (double)__fmul_rn(s.w, qq.w);
    dq = gdn_warp_sum(dq);
    reinterpret_cast<float4 *>(state + (long)r * D)[lane] = s;
    if (lane == 0) a.out[hv + r] = __fmul_rn((float)dq, oscale);
    }
  }
  if (!__all_sync(0xffffffffu, finite) && lane == 0) report(a.status, kStatusNonfinite);
}

// ---- chunked prefill --------------------------------------------------------
//
// The chunkwise form of the recurrence (reference src/graph/prefill_gdn.rs:
// 223-456, generalised to 64-token chunks).  For a chunk of C tokens:
//   cum_t  = prod_{s<=t} decay_s,   P[t][j] = prod_{j<s<=t} decay_s
//   CK[t][j] = P[t][j] (k_j . k_t)  (j < t),  CQ[t][j] = P[t][j] (k_j . q_t)  (j <= t)
// and per state row r the deltas solve the unit lower-triangular system
//   delta_t + beta_t sum_{j<t} CK[t][j] delta_j = beta_t (v_rt - cum_t S_r.k_t),
// i.e. delta_r = M (v_r - cum o S_r K^T) with M = (I + diag(beta) CK)^-1 diag(beta).
//   o_rt    = (cum_t S_r.q_t + sum_{j<=t} CQ[t][j] delta_rj) / sqrt(d)
//   S_r    <- cum_{C-1} S_r + sum_j P[C-1][j] delta_rj k_j
// A prep kernel (one CTA per chunk) writes M, CQ, cum and P[C-1] to scratch;
// a scan kernel (one CTA per state-row group) walks the chunks in order with
// the state rows resident in shared memory.  binary32 throughout: the
// reference's own chunkwise form is checked against its sequential
// recurrence within 1e-3 + 1e-3 |ref| (docs/cpu-tiled-prefill.md:173-189).

constexpr int kChunk = 64;
constexpr int kGdnD = 128;
// shared-memory row strides: +4 floats keeps 16-byte loads of consecutive
// rows in distinct bank groups, +1 does the same for scalar column walks
constexpr int kKS = kGdnD + 4;
constexpr int kMS = kChunk + 1;
// 16-byte rows (a multiple of 4 floats, 4 banks apart) for tiles read as
// float4 along the row: the prep kernel's beta * CK and, in the prefetching
// scan, M, CQ and the delta-side tiles
constexpr int kMS4 = kChunk + 4;
// scratch floats per (sequence, head, chunk): M and CQ in rows of kMS4
// (the prefetching scan's tile layout, so that each arrives in one bulk
// copy), then cum and P[C-1]
constexpr int kChunkScratch = 2 * kChunk * kMS4 + 2 * kChunk;

struct GdnPrefillArgs {
  GdnBatchArgs g;
  int chunk;          // tokens per chunk (<= 64)
  int nchunks;        // ceil(T / chunk)
  float *scratch;     // [batch][heads][nchunks][kChunkScratch]
};

constexpr int kPrepThreads = 256;

__device__ __forceinline__ void cp_async16_zfill(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}


// grid (nchunks, heads, batch)
// Three CTAs per SM: the decay products and beta * CK reuse the K and Q
// space once the dots are in registers.
__global__ void __launch_bounds__(kPrepThreads, 3) gdn_chunk_prep_kernel(GdnPrefillArgs p) {
  constexpr int D = kGdnD, C = kChunk;
  extern __shared__ __align__(16) float sm[];
  float *K = sm;                 // [C][kKS]
  float *Q = K + C * kKS;        // [C][kKS]
  float *P = K;                  // [C][C+1]  decay products (padded), after the dots
  float *Bm = Q;                 // [C][kMS4]  beta * CK, after the dots
  float *cum = Q + C * kKS;      // [C]
  float *dec = cum + C;          // [C]
  float *bet = dec + C;          // [C]
  const GdnBatchArgs &a = p.g;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h % a.key_heads;
  const int t0 = c * p.chunk;
  const int n = min(p.chunk, a.T - t0);
  grid_dependency_wait();
  grid_dependents_launch();
  // the chunk's K and Q rows (zeros past the prompt's end) as asynchronous
  // copies, all in flight at once
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int t = i / (D / 4), col = i % (D / 4);
    const long off = (((long)b * a.T + t0 + min(t, n - 1)) * a.key_heads + kh) * D;
    cp_async16_zfill(K + t * kKS + 4 * col, a.k + off + 4 * col, t < n);
    cp_async16_zfill(Q + t * kKS + 4 * col, a.q + off + 4 * col, t < n);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int t = threadIdx.x; t < C; t += blockDim.x) {
    const long off = ((long)b * a.T + t0 + t) * a.heads + h;
    dec[t] = t < n ? a.decay[off] : 1.0f;
    bet[t] = t < n ? a.beta[off] : 0.0f;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    float d = 1.0f;
    for (int t = 0; t < C; ++t) {
      d = __fmul_rn(d, dec[t]);
      cum[t] = d;
    }
  }
  // CK (strict lower) scaled by beta_t into Bm, CQ (lower) to scratch
  float *scr = p.scratch + (((long)b * a.heads + h) * p.nchunks + c) * kChunkScratch;
  float *Mout = scr, *CQout = scr + C * kMS4, *cumout = scr + 2 * C * kMS4, *plast = cumout + C;
  {
    // register tiles: thread (ti, tj) owns t = ti + 16a, j = tj + 16b; the
    // dots keep the one-output-per-thread accumulation order
    constexpr int TA = 4;
    const int ti = threadIdx.x / 16, tj = threadIdx.x % 16;
    float dkk[TA][TA], dkq[TA][TA];
#pragma unroll
    for (int ai = 0; ai < TA; ++ai)
#pragma unroll
      for (int bi = 0; bi < TA; ++bi) dkk[ai][bi] = dkq[ai][bi] = 0.0f;
#pragma unroll 2
    for (int x = 0; x < D / 4; ++x) {
      float4 kt[TA], qt[TA], kj[TA];
#pragma unroll
      for (int ai = 0; ai < TA; ++ai) {
        kt[ai] = reinterpret_cast<const float4 *>(K + (ti + 16 * ai) * kKS)[x];
        qt[ai] = reinterpret_cast<const float4 *>(Q + (ti + 16 * ai) * kKS)[x];
        kj[ai] = reinterpret_cast<const float4 *>(K + (tj + 16 * ai) * kKS)[x];
      }
#pragma unroll
      for (int ai = 0; ai < TA; ++ai)
#pragma unroll
        for (int bi = 0; bi <= ai; ++bi) {
          // bi > ai puts every j above every t: those dots are never used
          const float4 u = kj[bi], w = kt[ai], z = qt[ai];
          dkk[ai][bi] = fmaf(u.x, w.x, fmaf(u.y, w.y, fmaf(u.z, w.z, fmaf(u.w, w.w, dkk[ai][bi]))));
          dkq[ai][bi] = fmaf(u.x, z.x, fmaf(u.y, z.y, fmaf(u.z, z.z, fmaf(u.w, z.w, dkq[ai][bi]))));
        }
    }
    __syncthreads();  // K and Q are read: their space takes P and Bm
    // P[t][j] = P[t][j+1] * decay_{j+1}, P[t][t] = 1 (reference order)
    for (int t = threadIdx.x; t < C; t += blockDim.x) {
      float pr = 1.0f;  // the chain in a register, each product stored once
      P[t * (C + 1) + t] = pr;
      for (int j = t - 1; j >= 0; --j) {
        pr = __fmul_rn(pr, dec[j + 1]);
        P[t * (C + 1) + j] = pr;
      }
      for (int j = t + 1; j < C; ++j) P[t * (C + 1) + j] = 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int ai = 0; ai < TA; ++ai)
#pragma unroll
      for (int bi = 0; bi < TA; ++bi) {
        const int t = ti + 16 * ai, j = tj + 16 * bi;
        float ck = 0.0f, cq = 0.0f;
        if (j <= t && t < n) {
          const float pr = P[t * (C + 1) + j];
          cq = pr * dkq[ai][bi];
          if (j < t) ck = pr * dkk[ai][bi];
        }
        Bm[t * kMS4 + j] = bet[t] * ck;
        CQout[t * kMS4 + j] = cq;
      }
  }
  for (int t = threadIdx.x; t < C; t += blockDim.x) {
    cumout[t] = cum[t];
    plast[t] = P[(n - 1) * (C + 1) + t];
  }
  __syncthreads();
  // T = (I + Bm)^-1 (unit lower triangular): thread j < C holds column j in
  // registers, T[t][j] = -sum_{k<t} Bm[t][k] T[k][j] in k order (the terms
  // k < j add zeros to the zero start, so the sum is the one over
  // j <= k < t); then M = T diag(beta).  Unrolled, a row's chain overlaps the
  // rows before it, and Bm is read four entries per (broadcast) load.
  if (threadIdx.x < C) {
    const int j = threadIdx.x;
    float col[C];
#pragma unroll
    for (int t = 0; t < C; ++t) col[t] = t == j ? 1.0f : 0.0f;
#pragma unroll
    for (int t = 1; t < C; ++t) {
      float s = 0.0f;
#pragma unroll
      for (int k4 = 0; k4 < t; k4 += 4) {
        const float4 bm = *reinterpret_cast<const float4 *>(Bm + t * kMS4 + k4);
        s = fmaf(bm.x, col[k4], s);
        if (k4 + 1 < t) s = fmaf(bm.y, col[k4 + 1], s);
        if (k4 + 2 < t) s = fmaf(bm.z, col[k4 + 2], s);
        if (k4 + 3 < t) s = fmaf(bm.w, col[k4 + 3], s);
      }
      if (t > j) col[t] = -s;
    }
    const float bj = bet[j];
#pragma unroll
    for (int t = 0; t < C; ++t) Mout[t * kMS4 + j] = col[t] * bj;
  }
}

__host__ __device__ constexpr size_t gdn_prep_smem() {
  static_assert(kChunk * (kChunk + 1) <= kChunk * kKS && kChunk * kMS4 <= kChunk * kKS,
                "P and Bm fit the K and Q space");
  return (size_t)(2 * kChunk * kKS + 3 * kChunk) * 4;
}

// Scan over the chunks of one (sequence, head) for kScanR state rows.
// grid (128 / kScanR, heads, batch), kScanThreads threads.  In each chunk the
// lower threads form the tiles (thread mappings at each phase) while the
// upper half issues the next chunk's K, Q and V asynchronous copies into a
// second buffer; the next chunk's M, CQ, cum and P[C-1] arrive by bulk
// copies on an mbarrier once the current chunk's outputs are formed.  Small
// row groups measured faster than 64-row groups at every batch (per row and
// chunk the tiles and copies overlap better), so every batch uses them.
constexpr int kScanThreads = 512;
constexpr int kScanR = 16;

__host__ __device__ constexpr size_t gdn_chunk_scan_smem() {
  // S[R][D], two K, Q [C][kKS] and V [C][R], M, CQ [C][kMS4], KD, QD, DL
  // [R][kMS4], two cum/plast [2][C]
  return (size_t)(kScanR * kGdnD + 2 * (2 * kChunk * kKS + kChunk * kScanR) + 2 * kChunk * kMS4 +
                  3 * kScanR * kMS4 + 2 * 2 * kChunk) *
         4;
}

__global__ void __launch_bounds__(kScanThreads, 1) gdn_chunk_scan_kernel(GdnPrefillArgs p) {
  constexpr int D = kGdnD, C = kChunk, R = kScanR;
  // row strides of M, CQ (MS) and KD, QD, DL (CP): 16-byte rows, read as
  // float4 along the row
  constexpr int MS = kMS4, CP = kMS4;
  extern __shared__ __align__(16) float sm[];
  float *S = sm;                          // [R][D]
  float *Kb = S + R * D;                  // [2][C][kKS]
  float *Qb = Kb + 2 * C * kKS;           // [2][C][kKS]
  float *Vb = Qb + 2 * C * kKS;           // [2][C][R]
  float *M = Vb + 2 * C * R;              // [C][MS]
  float *CQ = M + C * MS;                 // [C][MS]
  float *KD = CQ + C * MS;                // [R][CP]
  float *QD = KD + R * CP;                // [R][CP]
  float *DL = QD + R * CP;                // [R][CP]  deltas
  float *cumb = DL + R * CP;              // [2][2][C]: cum, then plast
  const GdnBatchArgs &a = p.g;
  const int g = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h % a.key_heads;
  const int r0 = g * R;
  const int tid = threadIdx.x;
  grid_dependency_wait();
  grid_dependents_launch();
  float *state = a.state + ((long)b * a.heads + h) * D * D + (long)r0 * D;
  for (int i = tid; i < R * D / 4; i += blockDim.x)
    reinterpret_cast<float4 *>(S)[i] = reinterpret_cast<const float4 *>(state)[i];
  // chunk c's K and Q rows and V slice into buffer `buf` (zeros past the
  // prompt's end), as asynchronous copies committed as one group by threads
  // first, first + stride, ... (with prefetch the upper half of the CTA,
  // which is idle while the lower one forms the state dots)
  auto issue = [&](int c, int buf, int first, int stride) {
    const int t0 = c * p.chunk, n = min(p.chunk, a.T - t0);
    float *K = Kb + buf * C * kKS, *Q = Qb + buf * C * kKS, *V = Vb + buf * C * R;
    for (int i = first; i < C * D / 4; i += stride) {
      const int t = i / (D / 4), col = i % (D / 4);
      const long off = (((long)b * a.T + t0 + min(t, n - 1)) * a.key_heads + kh) * D;
      cp_async16_zfill(K + t * kKS + 4 * col, a.k + off + 4 * col, t < n);
      cp_async16_zfill(Q + t * kKS + 4 * col, a.q + off + 4 * col, t < n);
    }
    for (int i = first; i < C * R / 4; i += stride) {
      const int t = i / (R / 4), q4 = i % (R / 4);
      const long off = (((long)b * a.T + t0 + min(t, n - 1)) * a.heads + h) * D + r0;
      cp_async16_zfill(V + t * R + 4 * q4, a.v + off + 4 * q4, t < n);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // With prefetch, chunk c's M, CQ, cum and P[C-1] arrive by three bulk
  // copies (the scratch holds them in the tile layout) into M, CQ and
  // cum/plast buffer `buf`, completing on sbar; M and CQ are free once the
  // chunk before has formed its outputs.
  __shared__ __align__(8) uint64_t sbar;
  auto issue_scr = [&](int c, int buf) {
    if (tid == 0) {
      const float *scr = p.scratch + (((long)b * a.heads + h) * p.nchunks + c) * kChunkScratch;
      mbar_arrive_expect_tx(&sbar, (2 * C * MS + 2 * C) * 4);
      fence_proxy_async_smem();
      bulk_g2s(M, scr, C * MS * 4, &sbar);
      bulk_g2s(CQ, scr + C * kMS4, C * MS * 4, &sbar);
      bulk_g2s(cumb + buf * 2 * C, scr + 2 * C * kMS4, 2 * C * 4, &sbar);
    }
  };
  if (tid == 0) {
    mbar_init(&sbar, 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (p.nchunks > 0) {
    if (tid >= kScanThreads / 2) issue(0, 0, tid - kScanThreads / 2, kScanThreads / 2);
    issue_scr(0, 0);
  }
  const float oscale = 1.0f / sqrtf((float)D);
  bool finite = true;
  int stalled = -1;  // the chunk whose copies never completed
  for (int c = 0; c < p.nchunks; ++c) {
    const int t0 = c * p.chunk;
    const int n = min(p.chunk, a.T - t0);
    const int buf = c & 1;
    __syncthreads();
    // this chunk's K, Q, V (copied by the upper half during the chunk before)
    // and M, CQ, cum, P[C-1] (bulk copies)
    if (tid >= kScanThreads / 2) asm volatile("cp.async.wait_group 0;" ::: "memory");
    const bool ok = mbar_wait_bounded(&sbar, c & 1, a.status);
    if (!__syncthreads_and(ok)) {
      stalled = c;
      break;
    }
    const float *K = Kb + buf * C * kKS, *Q = Qb + buf * C * kKS, *V = Vb + buf * C * R;
    const float *cum = cumb + buf * 2 * C, *plast = cum + C;
    // Every output keeps the accumulation order of the one-output-per-thread
    // form (so a sequence's result does not depend on its batch).
    // KD[r][t] = S_r . k_t, QD[r][t] = S_r . q_t: thread u < 128 owns rows
    // 8g..8g+7 (g = u / 64) of token u % 64
    // (each K/Q row read by 2 warps, each S row load shared by K and Q),
    // while the upper half of the CTA issues the next chunk's copies
    if (tid < 128) {
      const int g8 = 8 * (tid / 64), t = tid % 64;
      float dk[8], dq[8];
#pragma unroll
      for (int a8 = 0; a8 < 8; ++a8) dk[a8] = dq[a8] = 0.0f;
#pragma unroll 2
      for (int x = 0; x < D / 4; ++x) {
        const float4 u = reinterpret_cast<const float4 *>(K + t * kKS)[x];
        const float4 w = reinterpret_cast<const float4 *>(Q + t * kKS)[x];
#pragma unroll
        for (int a8 = 0; a8 < 8; ++a8) {
          const float4 sr = reinterpret_cast<const float4 *>(S + (g8 + a8) * D)[x];
          dk[a8] = fmaf(sr.x, u.x, fmaf(sr.y, u.y, fmaf(sr.z, u.z, fmaf(sr.w, u.w, dk[a8]))));
          dq[a8] = fmaf(sr.x, w.x, fmaf(sr.y, w.y, fmaf(sr.z, w.z, fmaf(sr.w, w.w, dq[a8]))));
        }
      }
#pragma unroll
      for (int a8 = 0; a8 < 8; ++a8) {
        const int r = g8 + a8;
        KD[r * CP + t] = V[t * R + r] - cum[t] * dk[a8];
        QD[r * CP + t] = dq[a8];
      }
    } else if (tid >= kScanThreads / 2 && c + 1 < p.nchunks) {
      issue(c + 1, buf ^ 1, tid - kScanThreads / 2, kScanThreads / 2);
    }
    __syncthreads();
    // delta[r][t] = sum_{j<=t} M[t][j] W[r][j]
    if (tid < 256) {
      const int g4 = 4 * (tid / 64), t = tid % 64;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      // four j per step (float4 along M's row and the W rows), the terms
      // j > t masked: the warp's tokens end at (t | 31)
      const int jend = (t | 31) + 1;
#pragma unroll 2
      for (int j4 = 0; j4 < jend; j4 += 4) {
        const float4 m4 = *reinterpret_cast<const float4 *>(M + t * MS + j4);
        float4 w4[4];
#pragma unroll
        for (int a4 = 0; a4 < 4; ++a4)
          w4[a4] = *reinterpret_cast<const float4 *>(KD + (g4 + a4) * CP + j4);
#pragma unroll
        for (int a4 = 0; a4 < 4; ++a4) {
          if (j4 <= t) acc[a4] = fmaf(m4.x, w4[a4].x, acc[a4]);
          if (j4 + 1 <= t) acc[a4] = fmaf(m4.y, w4[a4].y, acc[a4]);
          if (j4 + 2 <= t) acc[a4] = fmaf(m4.z, w4[a4].z, acc[a4]);
          if (j4 + 3 <= t) acc[a4] = fmaf(m4.w, w4[a4].w, acc[a4]);
        }
      }
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) DL[(g4 + a4) * CP + t] = t < n ? acc[a4] : 0.0f;
    }
    __syncthreads();
    // o[r][t] = (cum_t QD[r][t] + sum_{j<=t} CQ[t][j] delta[r][j]) / sqrt(d),
    // staged as [t][r] in the KD area (free now) for coalesced stores
    if (tid < 256) {
      const int g4 = 4 * (tid / 64), t = tid % 64;
      float acc[4];
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) acc[a4] = cum[t] * QD[(g4 + a4) * CP + t];
      const int jend = (t | 31) + 1;
#pragma unroll 2
      for (int j4 = 0; j4 < jend; j4 += 4) {
        const float4 c4 = *reinterpret_cast<const float4 *>(CQ + t * MS + j4);
        float4 d4[4];
#pragma unroll
        for (int a4 = 0; a4 < 4; ++a4)
          d4[a4] = *reinterpret_cast<const float4 *>(DL + (g4 + a4) * CP + j4);
#pragma unroll
        for (int a4 = 0; a4 < 4; ++a4) {
          if (j4 <= t) acc[a4] = fmaf(c4.x, d4[a4].x, acc[a4]);
          if (j4 + 1 <= t) acc[a4] = fmaf(c4.y, d4[a4].y, acc[a4]);
          if (j4 + 2 <= t) acc[a4] = fmaf(c4.z, d4[a4].z, acc[a4]);
          if (j4 + 3 <= t) acc[a4] = fmaf(c4.w, d4[a4].w, acc[a4]);
        }
      }
      float *O = KD;  // [C][R]
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) O[t * R + g4 + a4] = acc[a4] * oscale;
    } else if (tid < 384) {
      // S_r <- cum_last S_r + sum_j plast_j delta_rj k_j: thread u = tid - 256
      // owns rows 4 (u / 32) .. + 3 of columns 4 (u % 32) .. + 3, so each K
      // row is read by 4 warps.  It reads and writes only its own elements
      // of S (and the O phase none), so it runs beside the O phase.
      const int u = tid - 256, g4 = 4 * (u / 32), x4 = 4 * (u % 32);
      const float last = cum[n - 1];
      float acc[4][4];
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) {
        const float4 s0 = reinterpret_cast<const float4 *>(S + (g4 + a4) * D + x4)[0];
        acc[a4][0] = last * s0.x; acc[a4][1] = last * s0.y;
        acc[a4][2] = last * s0.z; acc[a4][3] = last * s0.w;
      }
      // four j per step (plast and the delta rows as float4), then the
      // j < n left over one at a time
      int j = 0;
#pragma unroll 2
      for (; j + 4 <= n; j += 4) {
        const float4 p4 = *reinterpret_cast<const float4 *>(plast + j);
        const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
        float dl[4][4];
        float4 kr[4];
#pragma unroll
        for (int a4 = 0; a4 < 4; ++a4) {
          const float4 d4 = *reinterpret_cast<const float4 *>(DL + (g4 + a4) * CP + j);
          dl[a4][0] = d4.x; dl[a4][1] = d4.y; dl[a4][2] = d4.z; dl[a4][3] = d4.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          kr[e] = reinterpret_cast<const float4 *>(K + (j + e) * kKS + x4)[0];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float kx[4] = {kr[e].x, kr[e].y, kr[e].z, kr[e].w};
#pragma unroll
          for (int a4 = 0; a4 < 4; ++a4) {
            const float cf = pj[e] * dl[a4][e];
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) acc[a4][c4] = fmaf(cf, kx[c4], acc[a4][c4]);
          }
        }
      }
      for (; j < n; ++j) {
        const float4 k0 = reinterpret_cast<const float4 *>(K + j * kKS + x4)[0];
        const float kx[4] = {k0.x, k0.y, k0.z, k0.w};
#pragma unroll
        for (int a4 = 0; a4 < 4; ++a4) {
          const float cf = plast[j] * DL[(g4 + a4) * CP + j];
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) acc[a4][c4] = fmaf(cf, kx[c4], acc[a4][c4]);
        }
      }
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) {
        float *sr = S + (g4 + a4) * D + x4;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          finite &= is_finite_f(acc[a4][c4]);
          sr[c4] = acc[a4][c4];
        }
      }
    }
    __syncthreads();
    if (c + 1 < p.nchunks) issue_scr(c + 1, buf ^ 1);  // M, CQ are free now
    for (int i = tid; i < R * C; i += blockDim.x) {
      const int t = i / R, r = i % R;  // r fastest: coalesced output stores
      if (t < n) a.out[(((long)b * a.T + t0 + t) * a.heads + h) * D + r0 + r] = KD[t * R + r];
    }
  }
  if (stalled >= 0) {
    // a chunk's bulk copies never completed (reported): wait for them once
    // more, again bounded, and for the asynchronous copies in flight, then
    // leave the state as it was
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (tid == 0) mbar_wait_bounded(&sbar, stalled & 1, a.status);
    __syncthreads();
    return;
  }
  __syncthreads();
  for (int i = tid; i < R * D / 4; i += blockDim.x)
    reinterpret_cast<float4 *>(state)[i] = reinterpret_cast<const float4 *>(S)[i];
  if (!__syncthreads_and(finite) && tid == 0) report(a.status, kStatusNonfinite);
}

}  // namespace prism
