// tp.cuh -- tensor-parallel sharding of the batched serving step.
//
// A rank owns a column slice (output rows) of every projection that feeds a
// per-head or per-row operation -- attention q/gate (query heads), k and v
// (the KV heads those query heads read), the Gated DeltaNet qkv / z / beta /
// alpha (its heads), FFN up and gate (256-row blocks of the intermediate) --
// and the matching row slice (input blocks) of the projections that leave
// them: attn_output, ssm_out and ffn_down.  Those three produce a partial
// sum of the full hidden vector on every rank, which the ranks all-reduce
// before the residual add.  The output head is split by vocabulary rows and
// the greedy token is the maximum of the ranks' (value, index) keys.
//
// The all-reduce runs over peer memory, fused into the kernels on either
// side of it:
//   * the row-parallel GEMM's epilogue stores its partial tile straight into
//     every rank's receive slot for this rank (P2P stores over NVLink /
//     NVSwitch), fences at system scope and bumps each rank's arrival
//     counter (gemm.cuh GemmPush);
//   * the next RMSNorm kernel waits (bounded) for its counter, sums the
//     ranks' partials in rank order, adds the residual and normalises.
// Every rank therefore sums the same values in the same order and holds
// bit-identical hidden states.  Two receive slots alternate between the
// attention/GDN exchange and the FFN exchange: a rank can be at most one
// exchange ahead of another (its next reduce needs the other's partial), so
// a slot is never overwritten before every rank has read it.  Counters only
// grow; an exchange's target is derived from the rank's completed-step count.
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
};

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

// This rank's exchange buffer: 256 B of counters (slot 0, slot 1, keys),
// two receive slots [ranks][M][hidden] f32, then the greedy keys [ranks][M].
struct TpExchange {
  static constexpr size_t kHead = 256;
  uint8_t *base = nullptr;
  size_t slot_bytes = 0, bytes = 0;
  int ranks = 1, M = 0, n = 0;
  uint8_t *peer[kMaxTp] = {};  // every rank's buffer as mapped here (own included)
  bool opened[kMaxTp] = {};    // peer[p] came from cudaIpcOpenMemHandle
  bool connected = false;
  unsigned long long *xstep = nullptr;  // steps completed on this rank, never reset

  void layout(int ranks_, int M_, int n_) {
    ranks = ranks_;
    M = M_;
    n = n_;
    slot_bytes = (size_t)ranks * M * n * sizeof(float);
    bytes = kHead + 2 * slot_bytes + (size_t)ranks * M * 8;
  }
  static unsigned long long *count(uint8_t *b, int i) {
    return reinterpret_cast<unsigned long long *>(b) + i;
  }
  float *slot(uint8_t *b, int s) const { return reinterpret_cast<float *>(b + kHead + s * slot_bytes); }
  unsigned long long *keys(uint8_t *b) const {
    return reinterpret_cast<unsigned long long *>(b + kHead + 2 * slot_bytes);
  }
  // the GEMM push of this rank's partial into slot s of every rank
  GemmPush push(int rank, int s) const {
    GemmPush g{};
    g.n = ranks;
    for (int p = 0; p < ranks; ++p) {
      g.dst[p] = slot(peer[p], s) + (size_t)rank * M * n;
      g.count[p] = count(peer[p], s);
    }
    return g;
  }
};

// An exchange's arrival target: (steps completed * per_step + index + 1) * inc.
struct TpWait {
  const unsigned long long *count;
  const unsigned long long *xstep;
  unsigned long long per_step, index, inc;
};

// Bounded wait (one thread) for an exchange; false when it expired or an
// earlier wait of this step already did (the step has failed: skip).
__device__ __forceinline__ bool tp_wait(const TpWait &w, unsigned *status) {
  if (*reinterpret_cast<volatile unsigned *>(status) & kStatusTimeout) return false;
  const unsigned long long target = (*w.xstep * w.per_step + w.index + 1ull) * w.inc;
  const unsigned long long t0 = global_timer_ns();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(w.count) : "memory");
    if (v >= target) break;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report(status, kStatusTimeout);
      return false;
    }
  }
  __threadfence_system();
  return true;
}

// All-reduce receive side fused with the next RMSNorm (one 256-thread CTA
// per token row): hidden = hidden + ((p_0 + p_1) + ... + p_{ranks-1}), then
// out = (hidden * scale) * w as rmsnorm_rows_kernel computes it.  With
// w == nullptr only the reduction runs.
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
  if (ok) {
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
  const double sum = block_sumsq_f64(x, n, red);
  const float mean = (float)(sum / (double)n);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  if ((!is_finite_f(scale) || !(scale > 0.0f)) && threadIdx.x == 0) report(status, kStatusNonfinite);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[row * n + i] = __fmul_rn(__fmul_rn(x[i], scale), nw[i]);
}

struct TpKeys {
  unsigned long long *dst[kMaxTp];    // rank p's key row for this rank
  unsigned long long *count[kMaxTp];  // rank p's key counter
};

// End of a tensor-parallel step (one CTA): send this rank's greedy keys
// (the maximum over its vocabulary slice) to every rank, wait for all of
// theirs, take the maximum in rank order -- the reference's lowest index
// among equal maxima, as the key encodes -- and advance every sequence.
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
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int p = 0; p < ranks; ++p) atomicAdd_system(push.count[p], 1ull);
    ok = tp_wait(w, status);
  }
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
