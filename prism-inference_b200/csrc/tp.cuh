// tp.cuh -- tensor-parallel sharding of the batched serving step.
//
// A rank owns a column slice (output rows) of every projection that feeds a
// per-head or per-row operation -- attention q/gate (query heads), k and v
// (the KV heads those query heads read), the Gated DeltaNet qkv / z / beta /
// alpha (its heads), FFN up and gate (256-row blocks of the intermediate)
// -- and the output head by vocabulary rows; the greedy token is the
// maximum of the ranks' (value, index) keys.  The projections that leave
// the heads and the FFN (attn_output, ssm_out, ffn_down) take one of two
// forms:
//
//  * exact (default): column-split too.  Each rank quantizes its heads' (or
//    FFN rows') output to Q8_K and stores the blocks straight into every
//    rank's token buffer (fused quantize + all-gather); every rank then
//    computes its slice of hidden rows over all K blocks and stores
//    residual + result into every rank's hidden state (fused GEMM epilogue +
//    all-gather).  Every value is computed exactly as on one GPU, so the
//    batch is bit-identical to the one-GPU batch and to the oracle.
//  * all-reduce: row-split (input blocks), as in Megatron-style tensor
//    parallelism.  Each rank's partial sum of the full hidden vector is
//    stored into a receive slot of every rank (fused GEMM epilogue); the
//    next RMSNorm sums the slots in rank order and adds the residual.  All
//    ranks agree bit for bit, but the cross-rank sums round differently
//    from the reference's sequential per-row chain, and the Q8_K
//    quantizers downstream turn those last-place differences into code
//    flips: outputs match the one-GPU batch only to a tolerance that widens
//    with depth.
//
// Every exchange is a producer storing over NVLink peer memory followed by
// a bounded counter wait (gemm.cuh TpWait / tp_publish).  The exchanges of a
// step are totally ordered across ranks (each waits for every rank's
// previous one), so one buffer per kind (two alternating slots for the
// all-reduce) is never overwritten before every rank has read it.
//
// Buffers are shared between the ranks' processes with CUDA IPC handles,
// which the host exchanges (one 64-byte handle per rank).
#pragma once

#include <vector>

#include "gemm.cuh"

namespace prism {

// The part of every linear a rank owns.
struct TpPlan {
  int rank = 0, size = 1;
  int qh0 = 0, qh1 = 0;  // attention query heads
  int kv0 = 0, kv1 = 0;  // KV heads read by those query heads
  int gh0 = 0, gh1 = 0;  // Gated DeltaNet heads (key head == value head)
  int fb0 = 0, fb1 = 0;  // FFN intermediate, in 256-row blocks
  int v0 = 0, v1 = 0;    // vocabulary rows of the output head (128-row tiles)
  int hr0 = 0, hr1 = 0;  // hidden rows of attn_output / ssm_out / ffn_down (exact form)
};

enum TpMode : int { kTpExact = 0, kTpAllReduce = 1 };

// Fills `p`; returns nullptr, or why the geometry cannot be split `size` ways.
inline const char *tp_plan(const prism_b200_qwen35_config &c, int rank, int size, TpPlan &p) {
  if (size < 1 || size > kMaxTp || rank < 0 || rank >= size)
    return "tensor-parallel size must be 1..8 and the rank below it";
  p.rank = rank;
  p.size = size;
  if (size == 1) {  // one rank owns everything, whatever the geometry
    p.qh1 = (int)c.heads;
    p.kv1 = (int)c.kv_heads;
    p.gh1 = (int)c.ssm_values;
    p.fb1 = (int)(c.ffn / 256);
    p.v1 = (int)c.vocab;
    p.hr1 = (int)c.hidden;
    return nullptr;
  }
  if (c.kv_heads == 0 || c.heads % c.kv_heads) return "query heads not a multiple of KV heads";
  if (c.heads % size) return "query heads not divisible by the tensor-parallel size";
  const int qpr = (int)c.heads / size, group = (int)(c.heads / c.kv_heads);
  if (qpr % group && group % qpr) return "a rank's query heads would straddle KV heads";
  if ((qpr * c.head_dim) % 256) return "a rank's attention output is not whole 256-blocks";
  p.qh0 = rank * qpr;
  p.qh1 = p.qh0 + qpr;
  p.kv0 = p.qh0 / group;
  p.kv1 = (p.qh1 - 1) / group + 1;
  if (c.ssm_groups != c.ssm_values)
    return "Gated DeltaNet sharding needs as many key heads as value heads";
  if (c.ssm_values % size) return "Gated DeltaNet heads not divisible by the tensor-parallel size";
  const int gpr = (int)c.ssm_values / size;
  if ((gpr * c.ssm_state) % 256) return "a rank's Gated DeltaNet output is not whole 256-blocks";
  p.gh0 = rank * gpr;
  p.gh1 = p.gh0 + gpr;
  if (c.ffn % 256 || (int)(c.ffn / 256) < size) return "FFN blocks fewer than ranks";
  const int nbf = (int)c.ffn / 256;
  p.fb0 = rank * nbf / size;
  p.fb1 = (rank + 1) * nbf / size;
  const int tiles = (int)((c.vocab + kGemmN - 1) / kGemmN);
  if (tiles < size) return "vocabulary smaller than one tile per rank";
  p.v0 = rank * tiles / size * kGemmN;
  p.v1 = std::min<int>((int)c.vocab, (rank + 1) * tiles / size * kGemmN);
  p.hr0 = (int)((long)rank * c.hidden / size);
  p.hr1 = (int)((long)(rank + 1) * c.hidden / size);
  return nullptr;
}

// Build a tiled weight (dst: dh-row tiles of nb units) from the rows
// rowmap[0..rows) of a tiled source (sh-row tiles of snb units), taking
// blocks [b0, b0 + nb) of each row; rows past `rows` are zero padding.  One
// thread per (tile, block, row); the unit layout is matvec.cuh's.
template <int KIND>
__global__ void gather_tiled_kernel(const uint8_t *__restrict__ src, int sh, int snb,
                                    const int *__restrict__ rowmap, int rows, int b0, int nb,
                                    int dh, int dtiles, uint8_t *__restrict__ dst) {
  const int SU = unit_bytes(KIND, sh), DU = unit_bytes(KIND, dh);
  const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long)dtiles * nb * dh) return;
  const int r = (int)(gid % dh);
  const long u = gid / dh;
  const int t = (int)(u / nb), b = (int)(u % nb);
  const int row = t * dh + r;
  uint8_t *du = dst + u * DU;
  const uint8_t *su = nullptr;
  int sr = 0;
  if (row < rows) {
    const int s = rowmap[row];
    su = src + ((long)(s / sh) * snb + b0 + b) * SU;
    sr = s % sh;
  }
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int c = 0; c < 4; ++c)
    reinterpret_cast<uint4 *>(du)[c * dh + r] =
        su ? reinterpret_cast<const uint4 *>(su)[c * sh + sr] : z;
  if (KIND == 35) {
    reinterpret_cast<uint16_t *>(du + 64 * dh)[r] =
        su ? reinterpret_cast<const uint16_t *>(su + 64 * sh)[sr] : (uint16_t)0;
  } else {
    reinterpret_cast<uint4 *>(du + 64 * dh)[r] =
        su ? reinterpret_cast<const uint4 *>(su + 64 * sh)[sr] : z;
    const uint16_t *sd = su ? reinterpret_cast<const uint16_t *>(su + 80 * sh) : nullptr;
    uint16_t *dd = reinterpret_cast<uint16_t *>(du + 80 * dh);
    dd[r] = sd ? sd[sr] : (uint16_t)0;
    dd[dh + r] = sd ? sd[sh + sr] : (uint16_t)0;
  }
}

// Row list of `ranges` ([first, end) row pairs of the source), in order.
inline std::vector<int> tp_rows(std::initializer_list<std::pair<int, int>> ranges) {
  std::vector<int> v;
  for (const auto &r : ranges)
    for (int i = r.first; i < r.second; ++i) v.push_back(i);
  return v;
}

// A new resident weight holding `rows` of `src`, blocks [b0, b0 + nb).  The
// allocation is appended to `allocs`.
inline cudaError_t tp_gather_weight(const DeviceWeight &src, const std::vector<int> &rows, int b0,
                                    int nb, int num_sms, std::vector<void *> &allocs,
                                    cudaStream_t s, DeviceWeight &out) {
  out = DeviceWeight{};
  out.kind = src.kind;
  out.rows = rows.size();
  out.cols = (uint64_t)nb * 256;
  out.nb = nb;
  out.h = choose_tile_height(src.kind, out.rows, out.cols, num_sms);
  out.ntiles = (int)((out.rows + out.h - 1) / out.h);
  const int unit = unit_bytes((int)src.kind, out.h);
  out.bytes = (uint64_t)out.ntiles * nb * unit;
  void *units = nullptr, *map = nullptr;
  cudaError_t e = cudaMalloc(&units, out.bytes);
  if (e != cudaSuccess) return e;
  allocs.push_back(units);
  out.units = static_cast<uint8_t *>(units);
  e = cudaMalloc(&map, rows.size() * sizeof(int));
  if (e != cudaSuccess) return e;
  e = cudaMemcpyAsync(map, rows.data(), rows.size() * sizeof(int), cudaMemcpyHostToDevice, s);
  const long threads = (long)out.ntiles * nb * out.h;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  if (e == cudaSuccess) {
    if (src.kind == 35)
      gather_tiled_kernel<35><<<grid, 256, 0, s>>>(src.units, src.h, src.nb,
                                                   static_cast<const int *>(map), (int)out.rows,
                                                   b0, nb, out.h, out.ntiles, out.units);
    else
      gather_tiled_kernel<10><<<grid, 256, 0, s>>>(src.units, src.h, src.nb,
                                                   static_cast<const int *>(map), (int)out.rows,
                                                   b0, nb, out.h, out.ntiles, out.units);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(map);
  return e;
}

// ---- the exchange ----------------------------------------------------------

// This rank's exchange buffer.  Counters (first 256 B): 0 hidden rows
// (exact) or slot 0 (all-reduce), 1 slot 1, 2 greedy keys, 3 gathered
// token blocks.  Then the all-reduce slots [2][ranks][M][hidden] f32, the
// greedy keys [ranks][M], and for the exact form the hidden state [M][hidden]
// and the gathered Q8_K token buffer.
struct TpExchange {
  static constexpr size_t kHead = 256;
  uint8_t *base = nullptr;
  int mode = kTpExact, ranks = 1, M = 0, n = 0, tok_nb = 0;
  size_t slot_bytes = 0, keys_off = 0, hidden_off = 0, tok_off = 0, bytes = 0;
  uint8_t *peer[kMaxTp] = {};  // every rank's buffer as mapped here (own included)
  bool opened[kMaxTp] = {};    // peer[p] came from cudaIpcOpenMemHandle
  bool connected = false;
  unsigned long long *xstep = nullptr;  // steps completed on this rank, never reset

  static size_t up(size_t v, size_t a) { return (v + a - 1) / a * a; }
  void layout(int mode_, int ranks_, int M_, int n_, int tok_nb_) {
    mode = mode_;
    ranks = ranks_;
    M = M_;
    n = n_;
    tok_nb = tok_nb_;
    slot_bytes = mode == kTpAllReduce ? (size_t)ranks * M * n * sizeof(float) : 0;
    keys_off = kHead + 2 * slot_bytes;
    hidden_off = up(keys_off + (size_t)ranks * M * 8, 256);
    tok_off = up(hidden_off + (mode == kTpExact ? (size_t)M * n * sizeof(float) : 0), 1024);
    bytes = tok_off + (mode == kTpExact ? token_q8k_bytes(M, tok_nb) : 0);
  }
  static unsigned long long *count(uint8_t *b, int i) {
    return reinterpret_cast<unsigned long long *>(b) + i;
  }
  float *slot(uint8_t *b, int s) const { return reinterpret_cast<float *>(b + kHead + s * slot_bytes); }
  unsigned long long *keys(uint8_t *b) const {
    return reinterpret_cast<unsigned long long *>(b + keys_off);
  }
  float *hidden(uint8_t *b) const { return reinterpret_cast<float *>(b + hidden_off); }
  uint8_t *tok(uint8_t *b) const { return b + tok_off; }
  // all-reduce: this rank's partial into slot s of every rank
  GemmPush push_partial(int rank, int s) const {
    GemmPush g{};
    g.n = ranks;
    g.ld = n;
    g.col = 0;
    for (int p = 0; p < ranks; ++p) {
      g.dst[p] = slot(peer[p], s) + (size_t)rank * M * n;
      g.count[p] = count(peer[p], s);
    }
    return g;
  }
  // exact: this rank's hidden rows [col, col + rows) into every rank's hidden
  GemmPush push_rows(int col) const {
    GemmPush g{};
    g.n = ranks;
    g.ld = n;
    g.col = col;
    for (int p = 0; p < ranks; ++p) {
      g.dst[p] = hidden(peer[p]);
      g.count[p] = count(peer[p], 0);
    }
    return g;
  }
};

// Quantize this rank's blocks of M token rows to Q8_K and store them into
// every rank's token buffer (fused quantize + all-gather): x is [M][nbl*256],
// its block b lands at block b0 + b of buffers carved for nbt blocks.  Each
// CTA then counts its (token, block) units on every rank's counter.
struct TpGather {
  TokenQ8K dst[kMaxTp];
  unsigned long long *count[kMaxTp];
  int ranks;
};

__global__ void __launch_bounds__(256) q8k_gather_kernel(const float *__restrict__ x, int M,
                                                         int nbl, int b0, int nbt, TpGather g,
                                                         unsigned *status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  grid_dependency_wait();
  grid_dependents_launch();
  const int units = M * nbl;
  if (warp < units) {
    const int m = warp / nbl, bl = warp % nbl;
    uint32_t w0, w1;
    int pair;
    float scale;
    quantize_token_unit(x, nbl, m, bl, lane, 0, w0, w1, pair, scale, status);
    for (int p = 0; p < g.ranks; ++p)
      store_token_unit(g.dst[p], nbt, m, b0 + bl, lane, w0, w1, pair, scale);
  }
  const int first = blockIdx.x * (blockDim.x >> 5);
  const int mine = max(0, min((int)(blockDim.x >> 5), units - first));
  tp_publish(g.count, g.ranks, (unsigned long long)mine);
}

// RMSNorm of each token row after an exchange (one 256-thread CTA per row):
// wait for the exchange; with ranks > 0 (all-reduce) first
// hidden += ((p_0 + p_1) + ... + p_{ranks-1}) over the slot's partials;
// then out = (hidden * scale) * w as rmsnorm_rows_kernel computes it.  With
// w == nullptr only the wait and the reduction run.
__global__ void __launch_bounds__(256)
    tp_reduce_norm_kernel(const float *slot, int ranks, int M, int n, TpWait w, float *hidden,
                          const float *nw, float eps, float *out, unsigned *status) {
  __shared__ double red[8];
  __shared__ int ok;
  grid_dependency_wait();
  grid_dependents_launch();
  if (threadIdx.x == 0) ok = tp_wait(w, status);
  __syncthreads();
  const long row = blockIdx.x;
  float *x = hidden + row * n;
  if (ok && ranks > 0) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float s = __ldcg(slot + row * n + i);
      for (int p = 1; p < ranks; ++p) s = __fadd_rn(s, __ldcg(slot + ((long)p * M + row) * n + i));
      const float v = __fadd_rn(x[i], s);
      if (!is_finite_f(v)) report(status, kStatusNonfinite);
      x[i] = v;
    }
  }
  __syncthreads();
  if (!nw) return;
  double sum = 0.0;
  {
    // block_sumsq_f64's order, over values other ranks may have stored
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float v = __ldcg(x + i);
      sum += (double)__fmul_rn(v, v);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = 0.0;
    for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) sum += red[wi];
  }
  const float mean = (float)(sum / (double)n);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  if ((!is_finite_f(scale) || !(scale > 0.0f)) && threadIdx.x == 0) report(status, kStatusNonfinite);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[row * n + i] = __fmul_rn(__fmul_rn(__ldcg(x + i), scale), nw[i]);
}

struct TpKeys {
  unsigned long long *dst[kMaxTp];    // rank p's key row for this rank
  unsigned long long *count[kMaxTp];  // rank p's key counter
};

// End of a tensor-parallel step (one CTA): send this rank's greedy keys
// (the maximum over its vocabulary slice) to every rank, wait for all of
// theirs, take the maximum -- the reference's lowest index among equal
// maxima, as the key encodes -- and advance every sequence.
__global__ void tp_finish_kernel(unsigned long long *keys, TpKeys push,
                                 const unsigned long long *recv, int ranks, TpWait w,
                                 uint32_t *tokens, int *pos, int B, int *step,
                                 unsigned long long *xstep, int greedy, unsigned *status) {
  __shared__ int ok;
  grid_dependency_wait();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const unsigned long long k = keys[b];
    for (int p = 0; p < ranks; ++p) push.dst[p][b] = k;
    keys[b] = 0ull;
  }
  tp_publish(push.count, ranks, 1ull);
  if (threadIdx.x == 0) ok = tp_wait(w, status);
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    if (greedy && ok) {
      unsigned long long best = 0ull;
      for (int p = 0; p < ranks; ++p) {
        const unsigned long long k = __ldcg(recv + (size_t)p * B + b);
        best = k > best ? k : best;
      }
      tokens[b] = 0xffffffffu - (unsigned)(best & 0xffffffffull);
    }
    pos[b] += 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *step += 1;
    *xstep += 1ull;
  }
}

}  // namespace prism
