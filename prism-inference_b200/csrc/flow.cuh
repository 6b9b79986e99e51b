// flow.cuh -- the Qwen3.5-style decode step as one persistent dataflow kernel.
//
// One cooperative launch per token: one CTA per SM, 16 compute warps plus one
// weight-streaming warp.  The step is a host-built list of phases
// (embedding; per layer the attention side and the FFN pair; the LM head).
//
// Synchronisation is carried by the data.  Every activation that crosses CTAs
// is a 64-bit word: binary32 value in the low half, a 32-bit tag in the high
// half.  The tag is (step epoch << 8) | k, where k is the index of the phase
// that wrote the word, so a reader that knows which phase produces its input
// polls those words until every one carries the expected tag and then uses
// the value it already holds.  There is no grid barrier, no counter and no
// fence between phases: a consumer waits for exactly the words it reads
// (a Gated DeltaNet head for its own q/k/v channels, a projection for the
// whole input vector), one L2 round trip after the last producer's store.
// Words are stored and loaded with .relaxed.gpu operations, so each 64-bit
// word is observed whole.  A buffer is rewritten only after every reader of
// its previous contents is done: a phase's readers finish reading before the
// phase's own outputs exist, and the next writer of a buffer transitively
// needs those outputs.
//
// The weights never wait for data: the streaming warp walks the same phase
// list and copies this CTA's weight tiles, phase after phase, into a
// shared-memory ring with bulk copies, as far ahead as the ring allows.  Each
// projection phase gives a CTA a contiguous range of tiles, so its copies are
// contiguous in HBM.  The compute warps stage the Q8_K activation, run the
// unit dots on resident tiles, release the tiles' ring space, then run each
// row's chain.
//
// The arithmetic is that of the per-kernel path (matvec.cuh,
// model_kernels.cuh, gdn_slices_kernel): the same unit dots, binary32 chains,
// binary64 reductions in the same order and the same transcendentals, so the
// two paths give identical bits.
//
// Every wait is bounded (kWaitLimitNs).  A CTA that gives up raises the
// step's abort word and the timeout status, and every other wait checks the
// abort word, so the whole grid leaves within one wait limit.  Failures are
// made CTA-uniform by a vote before anyone acts on them; copies in flight
// are drained (bounded) before a CTA exits.
#pragma once

#include "common.cuh"
#include "matvec.cuh"
#include "model_kernels.cuh"
#include "gdn_decode.cuh"

namespace prism {

constexpr int kFWarps = 16;                 // compute warps
constexpr int kFThreads = kFWarps * 32;     // compute threads (named barrier 1)
constexpr int kFBlock = kFThreads + 32;     // + the weight-streaming warp
constexpr int kFRing = 144 * 1024;          // weight ring
constexpr int kFSlots = 64;                 // pieces in flight
constexpr int kFMaxNb = 48;                 // input blocks per projection (12288 values)
constexpr int kFActBytes = (kFMaxNb * (256 + 4 + 32 + 4) + 127) / 128 * 128;
constexpr int kFWorkBytes = 58 * 1024;      // staging, terms, GDN / attention scratch
constexpr int kFDescBytes = 1024;
constexpr int kFAttnMaxPos = 2048;          // attention: positions of one head's scores
constexpr int kFKChunk = 16;                // attention: cached K rows per copy job
constexpr int kFVDepth = 16;                // attention: V positions per share per copy job
constexpr int kFAttnSlots = 7;              // attention: 8 KB slots the copy jobs rotate through
constexpr int kFAttnSlot = 8192;
constexpr int kFPieceMax = 32 * 1024;       // bytes of one weight-stream piece (soft cap)
// shared-memory layout
constexpr int kFOffAct = kFRing;
constexpr int kFOffWork = kFOffAct + kFActBytes;
constexpr int kFOffDesc = kFOffWork + kFWorkBytes;           // [kFDescBufs] phase descriptors
constexpr int kFDescBufs = 4;              // descriptors prefetched kFDescBufs - 1 phases ahead
constexpr int kFOffBars = kFOffDesc + kFDescBufs * kFDescBytes;  // ring [kFSlots], desc [4], kv [4]
constexpr int kFOffMeta = kFOffBars + (kFSlots + 8) * 8;     // off/len [kFSlots], counters
constexpr int kFOffRed = kFOffMeta + kFSlots * 8 + 64;       // double [2][16] + float [16]
constexpr int kFOffRes = kFOffRed + 2 * 16 * 8 + 16 * 4 + 64;  // u64 [kFThreads] residual words
constexpr int kFOffTab = kFOffRes + kFThreads * 8;            // batch tile table [4][16] u32
constexpr int kFOffIssue = kFOffTab + 4 * kFWarps * 4;         // u64 [kFSlots] (traced steps)
constexpr int kFMaxPieces = 48;                               // weight-stream pieces per phase
constexpr int kFOffPieces = kFOffIssue + kFSlots * 8;         // count + [4][kFMaxPieces]
constexpr int kFSmemBytes = kFOffPieces + (4 + 4 * kFMaxPieces) * 4;
static_assert(kFSmemBytes <= 232448, "flow kernel shared memory");

enum FPhaseType : int { kFEmbed = 0, kFProj = 1, kFGdn = 2, kFAttn = 3 };
enum FPrologue : int { kFRms = 0, kFF32 = 1, kFGated = 2 };

// A projection phase: a group of weights sharing one input.
struct FProj {
  int count, nb, epi, prologue;
  int tile_start[kMaxGroup + 1];
  int ntiles;                        // tiles of the phase (the SwiGLU pair: per weight)
  int h[kMaxGroup], rows[kMaxGroup];
  int part[kMaxGroup];               // bytes of one tile of weight g
  int most[kMaxGroup];               // tiles per weight-stream piece of weight g
  const uint8_t *units[kMaxGroup];
  uint64_t *out[kMaxGroup];          // tagged outputs (the pair: up * silu(gate) in out[0])
  float *plain[kMaxGroup];           // optional plain binary32 copies of the outputs
  const uint64_t *in;                // tagged input vector [nb * 256]
  int in_k;
  const uint64_t *zs;                // kFGated: SiLU(z) [heads * head_dim], tagged
  int zs_k;
  const float *norm_w;               // kFRms: [nb * 256]; kFGated: [head_dim]
  const uint64_t *res;               // residual rows (tagged), or null
  int res_k;
  int heads, head_dim;               // kFGated geometry
  float eps;
  unsigned long long *argmax_key;    // kEpiArgmax
};

// A Gated DeltaNet layer: value head h over kGdnSlices CTAs of 16 state rows.
struct FGdn {
  const uint64_t *mixed, *z, *beta, *alpha;  // the projection phase's outputs
  int in_k;
  const float *conv_w, *dt_bias, *ssm_a;
  float *conv_state;                 // two buffers by position parity
  long conv_buf_stride;
  float *state;                      // [values][S][S]
  uint64_t *o, *zs;                  // pre-norm output, SiLU(z): [values * S], tagged
  int S, groups, values, conv_k;
  float eps;
};

// Gated full attention: query head h over kAttnSplit CTAs (positions split).
struct FAttn {
  const uint64_t *proj, *key, *value;  // [heads][2][hd] query|gate, [kv*hd], [kv*hd]
  int in_k;
  const float *q_norm, *k_norm;
  uint8_t *kcache, *vcache;          // binary16 rows [context][kv*hd] or Q8_0 records
  int q8;
  int heads, kv_heads, hd, rope_dim;
  int sections[3];
  float eps, theta_scale;
  uint64_t *sc;                      // [heads][ctx] scores of the cached positions, tagged
  int ctx;
  uint64_t *out;                     // [heads * hd] gated output, tagged
};

struct FEmbed {
  const uint8_t *units;
  int h, nb, vocab, n;
  uint64_t *hidden;
  float *plain;
};

struct alignas(16) FPhase {
  int type, k;
  FProj pr;
  FGdn gd;
  FAttn at;
  FEmbed em;
};
static_assert(sizeof(FPhase) <= kFDescBytes && sizeof(FPhase) % 16 == 0, "phase descriptor");

struct FlowArgs {
  const FPhase *phases;
  int nphases;
  StepState st;
  int write_greedy;
  unsigned *sync;        // [0] finished CTAs, [1] abort word, [2] step epoch
  unsigned long long *key;  // the LM head's greedy key while the step runs
  unsigned *status;
  unsigned long long *trace;  // optional: [16 * phase] CTA 0's globaltimer stamps
  unsigned long long *trace_cta;  // optional: [phase][CTA][4] inputs arrived, staged, end, planned
};

// ---- small helpers -------------------------------------------------------------

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// Barrier of the compute warps that also ANDs a predicate over them.
__device__ __forceinline__ bool csync_and(bool p) {
  int r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\tsetp.ne.s32 a, %1, 0;\n\t"
      "bar.red.and.pred b, 1, 512, a;\n\tselp.s32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"((int)p)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_word(uint64_t *p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t tagged(float v, uint32_t tag) {
  return ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
}
__device__ __forceinline__ uint64_t tagged_u(uint32_t v, uint32_t tag) {
  return ((uint64_t)tag << 32) | (uint64_t)v;
}
__device__ __forceinline__ bool has_tag(uint64_t w, uint32_t tag) {
  return (uint32_t)(w >> 32) == tag;
}
__device__ __forceinline__ float word_value(uint64_t w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ double word_pair_value(uint64_t lo, uint64_t hi) {
  return __longlong_as_double((long long)(((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo));
}

__device__ __forceinline__ uint32_t ld_acquire_cta(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(uint32_t *p, uint32_t v) {
  asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}

// 8-byte asynchronous copy global -> shared (not a register load, so a
// barrier does not wait for it); completed by cp_async_wait_all().
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most n of this thread's most recently committed groups are
// pending (n above 7 waits for more than asked, which is safe).
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

struct FlowCtl {
  unsigned *status;
  unsigned *abort;
};

__device__ __forceinline__ bool flow_aborted(const FlowCtl &c) {
  return *reinterpret_cast<volatile const unsigned *>(c.abort) != 0u;
}

__device__ __forceinline__ void flow_raise(const FlowCtl &c) {
  report(c.status, kStatusTimeout);
  atomicExch(c.abort, 1u);
}

// Called after a poll round that found a word not yet written: keeps the
// wait bounded (kWaitLimitNs) and leaves early when another CTA aborted.
// The abort word (a global load, a round trip during which nothing is
// polled) is consulted only once a wait has lasted kSpinAbortNs, longer
// than any wait of a step that runs normally.
constexpr unsigned long long kSpinAbortNs = 20000;
struct Spin {
  unsigned long long t0 = 0;
  int rounds = 0;
  __device__ __forceinline__ bool again(const FlowCtl &c) {
    if (rounds++ == 0) {
      t0 = global_timer_ns();
      return true;
    }
    if ((rounds & 31) == 0) {
      const unsigned long long waited = global_timer_ns() - t0;
      if (waited > kSpinAbortNs && flow_aborted(c)) return false;
      if (waited > kWaitLimitNs) {
        flow_raise(c);
        return false;
      }
    }
    return true;
  }
};

// Wait for one word; returns false on timeout / abort.
__device__ __forceinline__ bool wait_word(const uint64_t *p, uint32_t tag, uint64_t &w,
                                          const FlowCtl &c) {
  w = ld_word(p);
  Spin sp;
  while (!has_tag(w, tag)) {
    if (!sp.again(c)) return false;
    w = ld_word(p);
  }
  return true;
}

// Wait for the words *p[j], j < N, with every load in flight at once;
// their values into v[j].
template <int N>
__device__ __forceinline__ bool wait_each(const uint64_t *const (&p)[N], uint32_t tag,
                                          float (&v)[N], const FlowCtl &c) {
  uint64_t w[N];
#pragma unroll
  for (int j = 0; j < N; ++j) w[j] = ld_word(p[j]);
  Spin sp;
  for (;;) {
    bool all = true;
#pragma unroll
    for (int j = 0; j < N; ++j) all &= has_tag(w[j], tag);
    if (all) break;
    if (!sp.again(c)) return false;
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (!has_tag(w[j], tag)) w[j] = ld_word(p[j]);
  }
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = word_value(w[j]);
  return true;
}

// Wait for the n (<= N) words p[i0 + j*stride]; their values into v[j].
template <int N>
__device__ __forceinline__ bool wait_words(const uint64_t *p, int i0, int stride, int n,
                                           uint32_t tag, float (&v)[N], const FlowCtl &c) {
  uint64_t w[N];
#pragma unroll
  for (int j = 0; j < N; ++j) w[j] = j < n ? ld_word(p + i0 + j * stride) : tagged_u(0u, tag);
  Spin sp;
  for (;;) {
    bool all = true;
#pragma unroll
    for (int j = 0; j < N; ++j) all &= has_tag(w[j], tag);
    if (all) break;
    if (!sp.again(c)) return false;
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (j < n && !has_tag(w[j], tag)) w[j] = ld_word(p + i0 + j * stride);
  }
#pragma unroll
  for (int j = 0; j < N; ++j) v[j] = word_value(w[j]);
  return true;
}

// Binary64 sum over the compute warps in block_sum_f64's order for a
// 512-thread block; red holds >= 16 doubles.
__device__ __forceinline__ double fsum_f64(double v, double *red) {
  v = warp_sum_f64(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  csync();
  if (lane == 0) red[warp] = v;
  csync();
  double t = 0.0;
  for (int w = 0; w < kFWarps; ++w) t += red[w];
  return t;
}

// Two binary64 sums over the compute warps at once, each in fsum_f64's
// order; red holds >= 32 doubles.
__device__ __forceinline__ void fsum2_f64(double &a, double &b, double *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double x = __shfl_xor_sync(0xffffffffu, a, off);
    const double y = __shfl_xor_sync(0xffffffffu, b, off);
    a += x;
    b += y;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  csync();
  if (lane == 0) {
    red[warp] = a;
    red[16 + warp] = b;
  }
  csync();
  double ta = 0.0, tb = 0.0;
  for (int w = 0; w < kFWarps; ++w) {
    ta += red[w];
    tb += red[16 + w];
  }
  a = ta;
  b = tb;
}

__device__ __forceinline__ float fmax_f32(float v, float *red) {
  v = warp_max_f32(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  csync();
  if (lane == 0) red[warp] = v;
  csync();
  float t = red[0];
  for (int w = 1; w < kFWarps; ++w) t = fmaxf(t, red[w]);
  return t;
}

// This CTA's contiguous share [t0, t1) of T units of work.
__device__ __forceinline__ void flow_range(int T, int &t0, int &t1) {
  t0 = (int)((long)blockIdx.x * T / gridDim.x);
  t1 = (int)((long)(blockIdx.x + 1) * T / gridDim.x);
}

__device__ __forceinline__ int flow_group(const FProj &p, int t) {
  int g = 0;
#pragma unroll
  for (int i = 1; i < kMaxGroup; ++i)
    if (i < p.count && t >= p.tile_start[i]) g = i;
  return g;
}

// One piece of the weight stream: a run of consecutive tiles of one weight
// (the pair: the same tiles of up and of gate), at most most[g] tiles
// (about 32 KB, at least one tile, never more than a batch holds), starting
// at tile t of this CTA's range [t, t1).  One bulk copy per weight moves it:
// a copy's fixed cost on the SM's copy engine (about 0.1-0.2 us) makes
// small copies the stream's limit.
struct FPiece {
  int g, lt, nt;     // weight, its first local tile, tiles
  uint32_t part;     // bytes of one tile of one weight
  uint32_t bytes;    // ring bytes (the pair: both runs)
};
__device__ __forceinline__ FPiece piece_at(int count, const int *tile_start, const int *part,
                                           const int *most, bool pair, int ntiles, int t, int t1) {
  FPiece q;
  q.g = 0;
  if (!pair)
#pragma unroll
    for (int i = 1; i < kMaxGroup; ++i)
      if (i < count && t >= tile_start[i]) q.g = i;
  const int end = pair ? ntiles : tile_start[q.g + 1];
  q.lt = pair ? t : t - tile_start[q.g];
  q.part = (uint32_t)part[q.g];
  q.nt = min(min(t1, end) - t, most[q.g]);
  q.bytes = (uint32_t)q.nt * q.part * (pair ? 2u : 1u);
  return q;
}

// ---- ring state ------------------------------------------------------------------

struct FRing {
  uint8_t *data;
  uint64_t *bar;      // [kFSlots] piece arrivals
  uint32_t *off;      // [kFSlots] data offset of the piece
  uint32_t *len;      // [kFSlots] bytes the piece holds (padding + data)
  uint32_t *tail;     // bytes released by the consumer (monotonic)
  uint32_t *released; // pieces released by the consumer
  uint32_t *issued;   // pieces issued by the producer (written at its exit)
  uint32_t *issued_live;  // pieces issued so far (release after each issue)
  uint32_t *desc_done;    // phases the compute warps finished (release)
  uint32_t *desc_fetched; // descriptors the fetcher issued
  unsigned long long *issue_ts;  // [kFSlots] issue time of each piece (traced steps)
};

// The weight-streaming warp (lane 0): every projection phase's tiles of this
// CTA in phase order, each tile (the pair: both weights' tiles) as one
// piece, as ring space frees up.
template <int KIND>
__device__ void flow_producer(const FlowArgs &fa, const FRing &rg, const FlowCtl &c) {
  uint32_t head = 0, issued = 0;
  bool ok = true;
  // the phase's plan in registers: the waits below clobber memory, so
  // fields read through the descriptor would be reloaded from global memory
  // for every piece; the next phase's plan is loaded while this one issues
  struct Plan {
    const uint8_t *units[kMaxGroup];
    int tile_start[kMaxGroup + 1];
    int part[kMaxGroup], most[kMaxGroup];
    int type, epi, ntiles, count;
  };
  auto load_plan = [&](int p) {
    Plan q;
    const FPhase &ph = fa.phases[p];
    q.type = ph.type;
    q.epi = ph.pr.epi;
    q.ntiles = ph.pr.ntiles;
    q.count = ph.pr.count;
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      q.units[g] = ph.pr.units[g];
      q.part[g] = ph.pr.part[g];
      q.most[g] = ph.pr.most[g];
      q.tile_start[g] = ph.pr.tile_start[g];
    }
    q.tile_start[kMaxGroup] = ph.pr.tile_start[kMaxGroup];
    return q;
  };
  Plan next = load_plan(0);
  for (int p = 0; p < fa.nphases && ok; ++p) {
    const Plan pr = next;
    if (p + 1 < fa.nphases) next = load_plan(p + 1);
    if (pr.type != kFProj) continue;
    const bool pair = pr.epi == kEpiSwiglu;
    int t0, t1;
    flow_range(pr.ntiles, t0, t1);
    for (int t = t0; t < t1 && ok;) {
      const FPiece q = piece_at(pr.count, pr.tile_start, pr.part, pr.most, pair, pr.ntiles, t, t1);
      t += q.nt;
      const uint32_t bytes = q.bytes;
      uint32_t off = head % (uint32_t)kFRing;
      const uint32_t pad = off + bytes > (uint32_t)kFRing ? (uint32_t)kFRing - off : 0u;
      // wait for room: ring bytes and a free slot
      Spin sp;
      for (;;) {
        const uint32_t tail = ld_acquire_cta(rg.tail);
        const uint32_t rel = ld_acquire_cta(rg.released);
        if (head + pad + bytes - tail <= (uint32_t)kFRing && issued - rel < (uint32_t)kFSlots)
          break;
        if (!sp.again(c)) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
      if (!ok) break;
      fence_proxy_async_smem();  // released space was read through the generic proxy
      head += pad;
      off = head % (uint32_t)kFRing;
      const int slot = (int)(issued % kFSlots);
      rg.off[slot] = off;
      rg.len[slot] = pad + bytes;
      const uint32_t run = (uint32_t)q.nt * q.part;
      if (fa.trace) rg.issue_ts[slot] = global_timer_ns();
      mbar_arrive_expect_tx(&rg.bar[slot], bytes);
      bulk_g2s(rg.data + off, pr.units[q.g] + (size_t)q.lt * q.part, run, &rg.bar[slot]);
      if (pair)
        bulk_g2s(rg.data + off + run, pr.units[1] + (size_t)q.lt * q.part, run, &rg.bar[slot]);
      head += bytes;
      ++issued;
      st_release_cta(rg.issued_live, issued);
    }
  }
  *rg.issued = issued;
}

// ---- input staging -----------------------------------------------------------------

// Load the tagged input vector of n values into xs (shared), thread i taking
// indices i, i+512, ...; with `sumsq` also this thread's binary64 sum of
// squares in block_sumsq_f64's order.
__device__ __forceinline__ bool stage_words(const uint64_t *in, int n, uint32_t tag, float *xs,
                                            bool sumsq, double &s, const FlowCtl &c) {
  constexpr int kMax = kFMaxNb * 256 / kFThreads;  // 24
  const int i = threadIdx.x;
  const int cnt = i < n ? (n - i + kFThreads - 1) / kFThreads : 0;
  uint64_t w[kMax];
#pragma unroll
  for (int j = 0; j < kMax; ++j) w[j] = j < cnt ? ld_word(in + i + j * kFThreads) : tagged_u(0u, tag);
  Spin sp;
  for (;;) {
    bool all = true;
#pragma unroll
    for (int j = 0; j < kMax; ++j) all &= has_tag(w[j], tag);
    if (all) break;
    if (!sp.again(c)) return false;
#pragma unroll
    for (int j = 0; j < kMax; ++j)
      if (j < cnt && !has_tag(w[j], tag)) w[j] = ld_word(in + i + j * kFThreads);
  }
  s = 0.0;
#pragma unroll
  for (int j = 0; j < kMax; ++j)
    if (j < cnt) {
      const float v = word_value(w[j]);
      xs[i + j * kFThreads] = v;
      if (sumsq) s += (double)__fmul_rn(v, v);
    }
  return true;
}

// Q8_K of one 256-value block held 8 per lane (lane l: values 8l..8l+7),
// stored into the SoA activation: the same bits as q8k_quantize_regs +
// store_q8k_soa (Source rounding), with a shorter dependent chain.  The
// block maximum, the first value of largest magnitude, comes from a warp
// max reduction of this lane's first-largest magnitude, a ballot for the
// first lane holding it and one shuffle of its signed value; the block code
// sum from a warp add reduction.
__device__ __forceinline__ unsigned q8k_block_fast(const float (&v)[8], int lane, int b,
                                                   const MatvecSmem &L, uint8_t *act) {
  float best = 0.0f;
  bool finite = true;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    finite &= is_finite_f(v[i]);
    if (fabsf(v[i]) > fabsf(best)) best = v[i];
  }
  const unsigned mag = __float_as_uint(fabsf(best));
  const unsigned top = __reduce_max_sync(0xffffffffu, mag);
  const unsigned holders = __ballot_sync(0xffffffffu, mag == top);
  const float maximum = __shfl_sync(0xffffffffu, best, __ffs(holders) - 1);
  finite = __all_sync(0xffffffffu, finite);
  unsigned st = finite ? 0u : kStatusNonfinite;
  int q[8];
  float scale = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = 0;
  if (maximum != 0.0f && finite) {
    const float iscale = __fdiv_rn(-127.0f, maximum);
    if (!is_finite_f(iscale)) {
      st |= kStatusInvalid;
    } else {
      scale = __fdiv_rn(1.0f, iscale);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float r = fminf(rintf(__fmul_rn(v[i], iscale)), 127.0f);
        if (!(r >= -127.0f && r <= 127.0f)) {
          st |= kStatusInvalid;
          r = 0.0f;
        }
        q[i] = (int)r;
      }
    }
  }
  int own = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) own += q[i];
  const int pair_sum = own + __shfl_xor_sync(0xffffffffu, own, 1);
  const int total = __reduce_add_sync(0xffffffffu, own);
  int8_t *values = reinterpret_cast<int8_t *>(act + L.act_values()) + b * 256;
  const uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) |
                      ((uint32_t)(uint8_t)q[2] << 16) | ((uint32_t)(uint8_t)q[3] << 24);
  const uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) |
                      ((uint32_t)(uint8_t)q[6] << 16) | ((uint32_t)(uint8_t)q[7] << 24);
  reinterpret_cast<uint2 *>(values)[lane] = make_uint2(w0, w1);
  if ((lane & 1) == 0)
    reinterpret_cast<int16_t *>(act + L.act_sums())[b * 16 + (lane >> 1)] = (int16_t)pair_sum;
  if (lane == 0) {
    reinterpret_cast<float *>(act + L.act_scale())[b] = scale;
    reinterpret_cast<int *>(act + L.act_asum())[b] = total;
  }
  return st;
}

// Quantize xs[0, nb*256) into the Q8_K SoA activation at act (stage_from_f32's
// quantization, a block per warp), after RMSNorm scaling when `rms`.
// nw0/nw1: this lane's norm weights of block `warp`, loaded ahead of time.
__device__ __forceinline__ void quantize_staged(const float *xs, int nb, float scale,
                                                const float *norm_w, bool rms, uint8_t *act,
                                                unsigned *status, float4 nw0, float4 nw1) {
  const MatvecSmem L(nb, 32, 0, nb);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < nb; b += kFWarps) {
    const int base = b * 256 + lane * 8;
    float v[8];
    const float4 x0 = *reinterpret_cast<const float4 *>(xs + base);
    const float4 x1 = *reinterpret_cast<const float4 *>(xs + base + 4);
    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
    v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
    if (rms) {
      const float4 w0 = b == warp ? nw0 : *reinterpret_cast<const float4 *>(norm_w + base);
      const float4 w1 = b == warp ? nw1 : *reinterpret_cast<const float4 *>(norm_w + base + 4);
      const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), w[j]);
    }
    const unsigned st = q8k_block_fast(v, lane, b, L, act);
    if (st && lane == 0) report(status, st);
  }
}

// ---- phases ------------------------------------------------------------------------

__device__ __forceinline__ uint32_t flow_tag(uint32_t ep, int k) { return (ep << 8) | (uint32_t)k; }

template <int KIND>
__device__ void flow_embed(const FEmbed &e, const StepState &st, int pos, uint32_t tag,
                           unsigned *status) {
  const uint32_t token = st.tokens[pos];
  const bool valid = token < (uint32_t)e.vocab;
  if (!valid && blockIdx.x == 0 && threadIdx.x == 0) report(status, kStatusInvalid);
  int i0, i1;
  flow_range(e.n, i0, i1);
  for (int i = i0 + (int)threadIdx.x; i < i1; i += kFThreads) {
    const float v = valid ? decode_tiled<KIND>(e.units, e.h, e.nb, (int)token, i) : 0.0f;
    st_word(e.hidden + i, tagged(v, tag));
    if (e.plain) e.plain[i] = v;
  }
}

// A projection phase.  `cons` is the number of ring pieces consumed so far
// (the same in every compute thread).
template <int KIND>
__device__ bool flow_proj(const FProj &p, const FRing &rg, uint8_t *smem, uint32_t ep,
                          uint32_t tag, int &cons, const FlowCtl &c, unsigned long long *tr,
                          unsigned long long *ts, unsigned long long *trace_all) {
  int t0, t1;
  flow_range(p.ntiles, t0, t1);
  if (t0 >= t1) return true;
  const bool pair = p.epi == kEpiSwiglu;
  const int nb = p.nb, n = nb * 256, upt = pair ? 2 * nb : nb;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t *act = smem + kFOffAct;
  float *work = reinterpret_cast<float *>(smem + kFOffWork);
  double *red = reinterpret_cast<double *>(smem + kFOffRed);
  // this CTA's pieces of the phase (the weight stream's order), laid out by
  // one thread while the others stage the input
  int *pl_n = reinterpret_cast<int *>(smem + kFOffPieces);
  int *pl_nt = pl_n + 4, *pl_g = pl_nt + kFMaxPieces, *pl_lt = pl_g + kFMaxPieces;
  uint32_t *pl_bytes = reinterpret_cast<uint32_t *>(pl_lt + kFMaxPieces);
  // pl_n[0]: first piece of the current batch, [1] its pieces, [2] its
  // tiles, [3] pieces in the list
  uint32_t *tb_off_ = reinterpret_cast<uint32_t *>(smem + kFOffTab);
  uint32_t byte_cap = 0;
  // Plan the batch that starts at piece i0 (consumed pieces: cons) and lay
  // out its tile table: batches are runs of whole pieces, all of them when
  // the ring holds the phase's pieces together (they streamed during
  // earlier phases), else runs that leave room for the next batch; at most
  // one tile per compute warp.  Offsets are known once the stream issued the
  // pieces; their data is awaited separately.  Last thread only.
  auto plan = [&](int i0, int cons_at) -> bool {
    const int n = pl_n[3];
    int i1 = i0, ntl = 0;
    uint32_t bb = 0;
    while (i1 < n) {
      const int nt = pl_nt[i1];
      if (i1 > i0 && (ntl + nt > kFWarps || bb + pl_bytes[i1] > byte_cap)) break;
      ntl += nt;
      bb += pl_bytes[i1];
      ++i1;
    }
    const int np = i1 - i0;
    bool ok = true;
    if (np) {
      Spin sp;
      while ((int)(ld_acquire_cta(rg.issued_live) - (uint32_t)cons_at) < np) {
        if (!sp.again(c)) {
          ok = false;
          break;
        }
      }
      int k = 0;
      for (int i = 0; i < np && ok; ++i) {
        const uint32_t base = rg.off[(cons_at + i) % kFSlots];  // past any wrap padding
        const int nt = pl_nt[i0 + i], g = pl_g[i0 + i], lt = pl_lt[i0 + i];
        const uint32_t part = (uint32_t)p.part[g];
        for (int j = 0; j < nt; ++j, ++k) {
          tb_off_[k] = base + (uint32_t)j * part;
          tb_off_[kFWarps + k] = base + (uint32_t)(nt + j) * part;
          reinterpret_cast<int *>(tb_off_)[2 * kFWarps + k] = g;
          reinterpret_cast<int *>(tb_off_)[3 * kFWarps + k] = lt + j;
        }
      }
    }
    pl_n[0] = i0;
    pl_n[1] = np;
    pl_n[2] = ntl;
    return ok;
  };
  bool plan_ok = true;
  if (tid == kFThreads - 1) {
    int n = 0;
    uint32_t total = 0, maxpiece = 0;
    for (int t = t0; t < t1 && n < kFMaxPieces; ++n) {
      const FPiece q = piece_at(p.count, p.tile_start, p.part, p.most, pair, p.ntiles, t, t1);
      pl_nt[n] = q.nt;
      pl_g[n] = q.g;
      pl_lt[n] = q.lt;
      pl_bytes[n] = q.bytes;
      total += q.bytes;
      maxpiece = max(maxpiece, q.bytes);
      t += q.nt;
    }
    pl_n[3] = n;
    byte_cap = total + maxpiece <= (uint32_t)kFRing ? total : ((uint32_t)kFRing - maxpiece) / 2;
    plan_ok = plan(0, cons);
    if (ts) ts[3] = global_timer_ns();
  }

  // 1. the Q8_K activation
  if (p.prologue == kFGated) {
    // o and SiLU(z) per head, the gated norm into y (one warp per head,
    // gated_heads_norm's order), then the quantization of y
    const int S = p.head_dim;  // 128
    float *y = work;
    const uint32_t itag = flow_tag(ep, p.in_k), ztag = flow_tag(ep, p.zs_k);
    float nw[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) nw[q] = p.norm_w[32 * q + lane];
    bool ok = true;
    for (int h = warp; h < p.heads && ok; h += kFWarps) {
      float o[4], g[4];
      {
        // the head's outputs and SiLU(z) words, all eight loads in flight
        uint64_t w[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          w[q] = ld_word(p.in + h * S + 32 * q + lane);
          w[4 + q] = ld_word(p.zs + h * S + 32 * q + lane);
        }
        Spin sp;
        for (;;) {
          bool all = true;
#pragma unroll
          for (int q = 0; q < 4; ++q) all &= has_tag(w[q], itag) && has_tag(w[4 + q], ztag);
          if (all) break;
          if (!sp.again(c)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (!has_tag(w[q], itag)) w[q] = ld_word(p.in + h * S + 32 * q + lane);
            if (!has_tag(w[4 + q], ztag)) w[4 + q] = ld_word(p.zs + h * S + 32 * q + lane);
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          o[q] = word_value(w[q]);
          g[q] = word_value(w[4 + q]);
        }
      }
      ok = __all_sync(0xffffffffu, ok);  // the warp's shuffles below need every lane
      if (!ok) break;
      double t = 0.0;
#pragma unroll
      for (int q = 0; q < 4; ++q) t += warp_sum_f64((double)__fmul_rn(o[q], o[q]));
      const float mean = (float)(t / (double)S);
      const float nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float normed = __fmul_rn(__fmul_rn(o[q], nscale), nw[q]);
        y[h * S + 32 * q + lane] = __fmul_rn(normed, g[q]);
      }
    }
    if (!csync_and(ok)) return false;
    if (ts && tid == 0) ts[0] = global_timer_ns();
    quantize_staged(y, nb, 1.0f, nullptr, false, act, c.status, float4(), float4());
  } else {
    float *xs = work;
    double s = 0.0;
    const bool rms = p.prologue == kFRms;
    // the norm weights do not depend on this step: load them first
    float4 nw0 = float4(), nw1 = float4();
    if (rms && warp < nb) {
      nw0 = *reinterpret_cast<const float4 *>(p.norm_w + warp * 256 + lane * 8);
      nw1 = *reinterpret_cast<const float4 *>(p.norm_w + warp * 256 + lane * 8 + 4);
    }
    const bool ok = stage_words(p.in, n, flow_tag(ep, p.in_k), xs, rms, s, c);
    if (!csync_and(ok)) return false;
    if (ts && tid == 0) ts[0] = global_timer_ns();
    float scale = 1.0f;
    if (rms) {
      // block_sumsq_f64: per-thread sums, warp butterfly, warps in order
      const double sum = fsum_f64(s, red);
      if (tr) tr[13] = global_timer_ns();
      const float mean = (float)(sum / (double)n);
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
      if ((!is_finite_f(scale) || !(scale > 0.0f)) && tid == 0) report(c.status, kStatusNonfinite);
    }
    if (tr) tr[14] = global_timer_ns();
    quantize_staged(xs, nb, scale, p.norm_w, rms, act, c.status, nw0, nw1);
    if (tr) tr[15] = global_timer_ns();
  }
  csync();
  if (tr) tr[1] = global_timer_ns();
  if (ts && tid == 0) ts[1] = global_timer_ns();

  const MatvecSmem L(nb, 32, 0, nb);
  const int8_t *values = reinterpret_cast<const int8_t *>(act + L.act_values());
  const float *ascale = reinterpret_cast<const float *>(act + L.act_scale());
  const int16_t *asums = reinterpret_cast<const int16_t *>(act + L.act_sums());
  const int *aasum = reinterpret_cast<const int *>(act + L.act_asum());
  float *terms = work;  // [batch tiles][upt][32]

  // 2. batches of whole pieces (planned by the last thread, see above)
  uint32_t *tb_off = reinterpret_cast<uint32_t *>(smem + kFOffTab);
  uint32_t *tb_off2 = tb_off + kFWarps;
  int *tb_g = reinterpret_cast<int *>(tb_off2 + kFWarps);
  int *tb_lt = tb_g + kFWarps;
  unsigned long long best = 0ull;
  bool first = true;
  for (;;) {
    const int np = pl_n[1], ntl = pl_n[2];
    if (np == 0) break;
    // the batch's pieces have landed: one thread waits, the vote tells the rest
    bool arrived = plan_ok;
    unsigned long long *tw = trace_all && first ? trace_all : nullptr;  // CTA 0, thread 511
    if (tid == kFThreads - 1) {
      if (tw) tw[8] = global_timer_ns();
      for (int i = 0; i < np && arrived; ++i) {
        const int slot = (cons + i) % kFSlots;
        arrived = mbar_wait_bounded(&rg.bar[slot], (unsigned)((cons + i) / kFSlots) & 1u, c.status);
      }
      if (tw) {
        tw[9] = global_timer_ns();
        tw[11] = rg.issue_ts[(cons + np - 1) % kFSlots];
        tw[12] = np;
      }
    }
    if (!csync_and(arrived)) {
      if (tid == 0) flow_raise(c);
      return false;
    }
    if (tr && first) tr[2] = global_timer_ns();
    // the chain thread of a tile row (warp = tile in the batch, lane = row);
    // its residual row comes by an asynchronous copy during the dots (a
    // register load in flight would hold the barriers until it returns)
    const int ck = warp;
    const int cg = ck < ntl ? tb_g[ck] : 0;
    const int ch = p.h[cg];
    const int corow = (ck < ntl ? tb_lt[ck] : 0) * ch + lane;
    const bool chain = ck < ntl && lane < ch && corow < p.rows[cg];
    uint64_t *resw_s = reinterpret_cast<uint64_t *>(smem + kFOffRes) + tid;
    const uint32_t rtag = flow_tag(ep, p.res_k);
    if (chain && p.res && !pair) cp_async8(resw_s, p.res + corow);
    const int tot = ntl * upt;
    for (int u = warp; u < tot; u += kFWarps) {
      const int k = u / upt, j = u - k * upt;
      const int H = p.h[tb_g[k]];
      const bool second = pair && j >= nb;
      const int b = second ? j - nb : j;
      const uint8_t *ud = rg.data + (second ? tb_off2[k] : tb_off[k]) + b * unit_bytes(KIND, H);
      float *out = terms + (k * upt + j) * 32;
      int dot, dot2;
      float term;
      if (H == 32)
        unit_terms<KIND, 32>(ud, values + b * 256, aasum[b], asums + b * 16, ascale[b], lane, dot,
                             dot2, term);
      else if (H == 16)
        unit_terms<KIND, 16>(ud, values + b * 256, aasum[b], asums + b * 16, ascale[b], lane, dot,
                             dot2, term);
      else
        unit_terms<KIND, 8>(ud, values + b * 256, aasum[b], asums + b * 16, ascale[b], lane, dot,
                            dot2, term);
      if (lane < H) out[lane] = term;
    }
    csync();
    if (tr && first) tr[3] = global_timer_ns();
    if (tid == 0) {
      // the batch's ring space is free again
      uint32_t rel = 0;
      for (int i = 0; i < np; ++i) rel += rg.len[(cons + i) % kFSlots];
      st_release_cta(rg.tail, *rg.tail + rel);
      st_release_cta(rg.released, (uint32_t)(cons + np));
    }
    cons += np;
    // the next batch is planned while the chains run (its table is free:
    // every thread read this batch's entries before the barrier above)
    if (tid == kFThreads - 1) plan_ok = plan(pl_n[0] + np, cons);
    bool ok = true;
    if (chain) {
      const float *tk = terms + ck * upt * 32;
      // the reference's chain: sum = 0; sum += term_b for b in order
      // (unrolled so that the loads run ahead of the dependent adds)
      float sum = 0.0f;
#pragma unroll 8
      for (int b = 0; b < nb; ++b) sum = __fadd_rn(sum, tk[b * 32 + lane]);
      const int r = corow;
      if (pair) {
        float gsum = 0.0f;
#pragma unroll 8
        for (int b = nb; b < 2 * nb; ++b) gsum = __fadd_rn(gsum, tk[b * 32 + lane]);
        const float hv = __fmul_rn(sum, silu_f(gsum));
        if (!is_finite_f(sum) || !is_finite_f(gsum)) report(c.status, kStatusNonfinite);
        st_word(p.out[0] + r, tagged(hv, tag));
        if (p.plain[0]) p.plain[0][r] = hv;
      } else {
        if (p.res) {
          cp_async_wait_all();
          uint64_t resw = *resw_s;
          if (!has_tag(resw, rtag)) ok = wait_word(p.res + r, rtag, resw, c);
          sum = __fadd_rn(word_value(resw), sum);
        }
        if (!is_finite_f(sum)) report(c.status, kStatusNonfinite);
        if (p.out[cg]) st_word(p.out[cg] + r, tagged(sum, tag));
        if (p.plain[cg]) p.plain[cg][r] = sum;
        if (p.epi == kEpiArgmax) {
          const unsigned long long key = argmax_key(sum, r);
          best = key > best ? key : best;
        }
      }
    }
    // the terms buffer is reused by the next batch; the plan is published
    if (!csync_and(ok)) return false;
    if (tr && first) tr[4] = global_timer_ns();
    first = false;
  }
  if (p.epi == kEpiArgmax) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0 && best) atomicMax(p.argmax_key, best);
  }
  return true;
}

// Gated DeltaNet layer: value head h over kGdnSlices CTAs of 16 state rows
// (run_gdn's arithmetic).  Writes the pre-norm output and SiLU(z) of its
// rows; the gated output norm runs in the out-projection's prologue.
__device__ bool flow_gdn(const FGdn &a, int pos, uint8_t *smem, uint32_t ep, uint32_t tag,
                         const FlowCtl &c) {
  constexpr int S = 128, R = S / kGdnSlices;
  if ((int)blockIdx.x >= a.values * kGdnSlices) return true;
  float *q = reinterpret_cast<float *>(smem + kFOffWork);  // [S]
  float *k = q + S;                                        // [S]
  float *v = k + S;                                        // [R]
  float *sdb = v + R;                                      // decay, beta
  double *red = reinterpret_cast<double *>(smem + kFOffRed);
  const int h = blockIdx.x / kGdnSlices, slice = blockIdx.x % kGdnSlices, r0 = slice * R;
  const int kh = h % a.groups, kw = a.groups * S, hist = a.conv_k - 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int parity = pos & 1;
  const float *hist_in = a.conv_state + parity * a.conv_buf_stride;
  float *hist_out = a.conv_state + (parity ^ 1) * a.conv_buf_stride;
  const uint32_t itag = flow_tag(ep, a.in_k);
  // this slice's state rows (written by the previous step): before the inputs
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  float *row = a.state + (long)h * S * S + (long)(r0 + warp) * S;
  if (warp < R) s = reinterpret_cast<const float4 *>(row)[lane];
  // 1. convolution + SiLU of the head's q, k channels and this slice's v
  bool ok = true;
  if (tid < 2 * S + R) {
    const int part = tid < S ? 0 : tid < 2 * S ? 1 : 2;
    const int j = part < 2 ? tid - part * S : r0 + (tid - 2 * S);
    const int ch = part == 0 ? kh * S + j : part == 1 ? kw + kh * S + j : 2 * kw + h * S + j;
    const float *hj = hist_in + (long)ch * hist;
    const float *cj = a.conv_w + (long)ch * a.conv_k;
    float hv[8];
    for (int i = 0; i < hist; ++i) hv[i] = hj[i];
    uint64_t w;
    ok = wait_word(a.mixed + ch, itag, w, c);
    const float projected = word_value(w);
    float sum = 0.0f;
    for (int i = 0; i < hist; ++i) sum = __fadd_rn(sum, __fmul_rn(hv[i], cj[i]));
    sum = __fadd_rn(sum, __fmul_rn(projected, cj[hist]));
    const float act = silu_f(sum);
    if (part == 0) q[j] = act;
    else if (part == 1) k[j] = act;
    else v[j - r0] = act;
    if (ok && (part == 2 || (h == kh && slice == 0))) {
      float *nj = hist_out + (long)ch * hist;
      for (int i = 0; i + 1 < hist; ++i) nj[i] = hv[i + 1];
      if (hist > 0) nj[hist - 1] = projected;
    }
  } else if (tid == 2 * S + R) {
    const uint64_t *const src[2] = {a.alpha + h, a.beta + h};
    float x[2];
    ok = wait_each<2>(src, itag, x, c);
    sdb[0] = recurrent_decay_f(x[0], a.dt_bias[h], a.ssm_a[h], c.status);
    sdb[1] = sigmoid_f(x[1]);
  } else if (tid >= 2 * S + R + 32 && tid < 2 * S + R + 32 + R) {
    // SiLU(z) of this slice's rows, for the out-projection's gated norm
    const int i = h * S + r0 + (tid - (2 * S + R + 32));
    uint64_t wz;
    ok = wait_word(a.z + i, itag, wz, c);
    if (ok) st_word(a.zs + i, tagged(silu_f(word_value(wz)), tag));
  }
  if (!csync_and(ok)) return false;
  // 2. L2 normalisation of q and k (the kernel's block-sum order)
  {
    const float xq = tid < S ? q[tid] : 0.0f;
    const float xk = tid < S ? k[tid] : 0.0f;
    // both sums in fsum_f64's order, sharing their barriers
    double sq = tid < S ? (double)__fmul_rn(xq, xq) : 0.0;
    double sk = tid < S ? (double)__fmul_rn(xk, xk) : 0.0;
    fsum2_f64(sq, sk, red);
    const float scq = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sq), a.eps));
    const float sck = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sk), a.eps));
    // each thread rewrites only the q[tid], k[tid] it read itself
    if (tid < S) {
      q[tid] = __fmul_rn(xq, scq);
      k[tid] = __fmul_rn(xk, sck);
    }
  }
  csync();
  // 3. this slice's state rows, one per warp
  const float decay = sdb[0], beta = sdb[1];
  const float oscale = __fdiv_rn(1.0f, __fsqrt_rn((float)S));
  if (warp < R) {
    const float4 kk = reinterpret_cast<const float4 *>(k)[lane];
    const float4 qq = reinterpret_cast<const float4 *>(q)[lane];
    s.x = __fmul_rn(decay, s.x);
    s.y = __fmul_rn(decay, s.y);
    s.z = __fmul_rn(decay, s.z);
    s.w = __fmul_rn(decay, s.w);
    double dk = (double)__fmul_rn(s.x, kk.x) + (double)__fmul_rn(s.y, kk.y) +
                (double)__fmul_rn(s.z, kk.z) + (double)__fmul_rn(s.w, kk.w);
    dk = warp_sum_f64(dk);
    const float delta = __fmul_rn(__fsub_rn(v[warp], (float)dk), beta);
    s.x = __fadd_rn(s.x, __fmul_rn(delta, kk.x));
    s.y = __fadd_rn(s.y, __fmul_rn(delta, kk.y));
    s.z = __fadd_rn(s.z, __fmul_rn(delta, kk.z));
    s.w = __fadd_rn(s.w, __fmul_rn(delta, kk.w));
    const bool finite =
        is_finite_f(s.x) && is_finite_f(s.y) && is_finite_f(s.z) && is_finite_f(s.w);
    double dq = (double)__fmul_rn(s.x, qq.x) + (double)__fmul_rn(s.y, qq.y) +
                (double)__fmul_rn(s.z, qq.z) + (double)__fmul_rn(s.w, qq.w);
    dq = warp_sum_f64(dq);
    reinterpret_cast<float4 *>(row)[lane] = s;
    if (lane == 0) st_word(a.o + h * S + r0 + warp, tagged(__fmul_rn((float)dq, oscale), tag));
    if (!__all_sync(0xffffffffu, finite) && lane == 0) report(c.status, kStatusNonfinite);
  }
  return true;
}

// RMSNorm(x)*w, RoPE and binary16 rounding (norm_rope_round's arithmetic)
// of the query (xq, weights wq) and the current key (xk, wk) over hd
// (== 256) values held one per thread, threads at or past hd contributing
// zeros; the two reductions share their barriers.  bq and bk are [hd]
// scratch.
__device__ __forceinline__ void flow_norm_rope_round2(float xq, float xk, const float *wq,
                                                      const float *wk, float eps, int hd,
                                                      int rope, const float *cs, float *bq,
                                                      float *bk, double *red, float &oq,
                                                      float &ok_) {
  const int i = threadIdx.x;
  double sq = i < hd ? (double)__fmul_rn(xq, xq) : 0.0;
  double sk = i < hd ? (double)__fmul_rn(xk, xk) : 0.0;
  fsum2_f64(sq, sk, red);
  const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(sq / (double)hd), eps)));
  const float sck = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn((float)(sk / (double)hd), eps)));
  if (i < hd) {
    bq[i] = __fmul_rn(__fmul_rn(xq, scq), wq[i]);
    bk[i] = __fmul_rn(__fmul_rn(xk, sck), wk[i]);
  }
  csync();
  float a = i < hd ? bq[i] : 0.0f, b = i < hd ? bk[i] : 0.0f;
  const int half = rope / 2;
  if (i < half) {
    a = __fsub_rn(__fmul_rn(bq[i], cs[2 * i]), __fmul_rn(bq[i + half], cs[2 * i + 1]));
    b = __fsub_rn(__fmul_rn(bk[i], cs[2 * i]), __fmul_rn(bk[i + half], cs[2 * i + 1]));
  } else if (i < rope) {
    const int j = i - half;
    a = __fadd_rn(__fmul_rn(bq[j], cs[2 * j + 1]), __fmul_rn(bq[i], cs[2 * j]));
    b = __fadd_rn(__fmul_rn(bk[j], cs[2 * j + 1]), __fmul_rn(bk[i], cs[2 * j]));
  }
  csync();
  oq = round_f16(a);
  ok_ = round_f16(b);
}

// Attention of query head h split over kAttnSplit CTAs (attention_decode_
// kernel's arithmetic and reduction orders; hd == 256).  CTA r scores its
// share of the cached positions and publishes the scores as tagged words;
// every CTA of the head then forms the softmax over all positions itself --
// the maximum, each share's binary64 total in the tree that attention_
// decode_kernel's block reduction gives it, the shares' totals in rank
// order -- and CTA r accumulates output dimensions [r*32, r*32 + 32) over
// every position: each share's binary64 partial sum in position order, the
// shares in rank order.  The same sums as the kernel with one exchange
// instead of three.  The K rows of the CTA's share and the V column slices
// of every position stream through shared memory by 16-byte asynchronous
// copies issued before the inputs are awaited.
constexpr int kFAttnHead = 15360;  // q, kc, vc, buf, cs, probabilities, trees, partials, gate
static_assert((4 * 256 + 64 + kFAttnMaxPos) * 4 + (64 + 8 + 8 * 32) * 8 + 32 * 4 <= kFAttnHead,
              "attention head area");
static_assert(kFAttnHead + kFAttnSlots * kFAttnSlot <= kFActBytes + kFWorkBytes,
              "attention slots fit the activation and work areas");
static_assert(kFKChunk * 512 <= kFAttnSlot && 8 * kFVDepth * 64 <= kFAttnSlot,
              "a binary16 K chunk or V chunk fills one slot");

// Two binary64 warp sums in warp_sum_f64's butterfly, interleaved.
__device__ __forceinline__ void warp_sum2_f64(double &a, double &b) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double x = __shfl_xor_sync(0xffffffffu, a, off);
    const double y = __shfl_xor_sync(0xffffffffu, b, off);
    a += x;
    b += y;
  }
}

__device__ bool flow_attn(const FAttn &a, int pos, uint8_t *smem, uint32_t ep, uint32_t tag,
                          const FlowCtl &c, unsigned long long *tr) {
  if ((int)blockIdx.x >= a.heads * kAttnSplit) return true;
  const int hd = a.hd;
  uint8_t *area = smem + kFOffAct;
  float *q = reinterpret_cast<float *>(area);  // [hd]
  float *kc = q + hd;
  float *vc = kc + hd;
  float *buf = vc + hd;
  float *cs = buf + hd;                        // [64]
  float *pr = cs + 64;                         // [kFAttnMaxPos] scores, exponentials, probabilities
  double *tw = reinterpret_cast<double *>(pr + kFAttnMaxPos);  // [share][warp] tree sums
  double *tot = tw + 64;                       // [share]
  double *part = tot + 8;                      // [share][32]
  float *gs = reinterpret_cast<float *>(part + 8 * 32);  // [32] gate
  double *red = reinterpret_cast<double *>(smem + kFOffRed);
  float *fred = reinterpret_cast<float *>(red + 32);
  const int rank = blockIdx.x % kAttnSplit, h = blockIdx.x / kAttnSplit;
  const int group = a.heads / a.kv_heads, kvh = h / group, kvw = a.kv_heads * hd;
  const int i = threadIdx.x, warp = i >> 5, lane = i & 31;
  const int per = (pos + kAttnSplit - 1) / kAttnSplit;
  const int lo = min(pos, rank * per), hi = min(pos, lo + per);
  const int rb = attn_row_bytes(hd, a.q8);
  const int dims = hd / kAttnSplit;  // 32: one Q8_0 block
  uint8_t *slots = area + kFAttnHead;  // [kFAttnSlots][kFAttnSlot]
  const int nk = (hi - lo + kFKChunk - 1) / kFKChunk;  // K jobs of this share
  const int nv = (per + kFVDepth - 1) / kFVDepth;      // V jobs (every share at once)
  const int njobs = nk + nv;
  auto krow = [&](int p) -> const uint8_t * {
    return a.q8 ? a.kcache + ((size_t)p * a.kv_heads + kvh) * rb
                : a.kcache + ((size_t)p * kvw + (size_t)kvh * hd) * 2;
  };
  // Copy job g (g < nk: K rows of the share; else V chunk g - nk: slot
  // r * kFVDepth + t holds position lo_r + k * kFVDepth + t of share r,
  // dimensions [rank*32, rank*32 + 32)) into slot g % kFAttnSlots, as one
  // cp.async group per thread: job g is group g of the phase.
  auto issue = [&](int g) {
    uint8_t *dst = slots + (size_t)(g % kFAttnSlots) * kFAttnSlot;
    if (g < nk) {
      const int p0 = lo + g * kFKChunk, count = min(kFKChunk, hi - p0), cpr = rb / 16;
      for (int j = i; j < count * cpr; j += kFThreads) {
        const int row = j / cpr, off = (j - row * cpr) * 16;
        cp_async16(dst + (size_t)row * rb + off, krow(p0 + row) + off);
      }
    } else {
      const int k = g - nk, cps = a.q8 ? 3 : 4;
      for (int j = i; j < 8 * kFVDepth * cps; j += kFThreads) {
        const int slot = j / cps, cp = j - slot * cps;
        const int r = slot / kFVDepth, t = slot - r * kFVDepth;
        const int lo_r = min(pos, r * per), hi_r = min(pos, lo_r + per);
        const int p = lo_r + k * kFVDepth + t;
        if (p >= hi_r) continue;
        if (a.q8) {
          const uint8_t *rec = a.vcache + ((size_t)p * a.kv_heads + kvh) * rb;
          if (cp < 2)
            cp_async16(dst + slot * 32 + cp * 16, rec + hd / 32 * 2 + rank * dims + cp * 16);
          else  // the aligned word holding block `rank`'s scale
            cp_async4(dst + 8 * kFVDepth * 32 + slot * 4, rec + (rank & ~1) * 2);
        } else {
          cp_async16(dst + slot * 64 + cp * 16,
                     a.vcache + ((size_t)p * kvw + (size_t)kvh * hd + rank * dims) * 2 + cp * 16);
        }
      }
    }
    cp_async_commit();
  };
  // every slot starts filling now; a consumed job's slot takes job g + slots
  int ng = min(njobs, kFAttnSlots);
  for (int g = 0; g < ng; ++g) issue(g);
  auto refill = [&](int g) {
    if (g + kFAttnSlots < njobs) {
      issue(g + kFAttnSlots);
      ++ng;
    }
  };
  if (i < a.rope_dim / 2) {
    float theta = (float)pos;
    for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, a.theta_scale);
    const float angle = i < 3 * a.sections[i % 3] ? theta : 0.0f;
    cs[2 * i] = cos_cr(angle);
    cs[2 * i + 1] = sin_cr(angle);
  }
  // inputs: query, current key and value (thread i < hd), the gate of this
  // CTA's output dimensions (threads hd .. hd + dims)
  const uint32_t itag = flow_tag(ep, a.in_k);
  float xq = 0.f, xk = 0.f, xv = 0.f;
  bool ok = true;
  if (i < hd) {
    const uint64_t *const src[3] = {a.proj + (long)h * 2 * hd + i, a.key + (long)kvh * hd + i,
                                    a.value + (long)kvh * hd + i};
    float x[3];
    ok = wait_each<3>(src, itag, x, c);
    xq = x[0];
    xk = x[1];
    xv = x[2];
  } else if (i < hd + dims) {
    uint64_t w = 0;
    ok = wait_word(a.proj + (long)(2 * h + 1) * hd + rank * dims + (i - hd), itag, w, c);
    gs[i - hd] = word_value(w);
  }
  if (!csync_and(ok)) return false;
  if (tr) tr[1] = global_timer_ns();
  float qv, kv_;
  flow_norm_rope_round2(xq, xk, a.q_norm, a.k_norm, a.eps, hd, a.rope_dim, cs, buf, vc, red, qv,
                        kv_);
  if (i < hd) {
    q[i] = qv;
    kc[i] = kv_;
    vc[i] = round_f16(xv);
    // the first CTA of the first query head of the group writes the cache row
    const bool writer = rank == 0 && h % group == 0;
    if (a.q8) {
      const long at = ((long)pos * a.kv_heads + kvh) * q8_0_record_bytes(hd);
      kc[i] = q8_0_roundtrip(kc[i], writer ? a.kcache + at : nullptr, hd, c.status);
      vc[i] = q8_0_roundtrip(vc[i], writer ? a.vcache + at : nullptr, hd, c.status);
    } else if (writer) {
      reinterpret_cast<uint16_t *>(a.kcache)[(long)pos * kvw + kvh * hd + i] =
          float_to_half_bits(kc[i]);
      reinterpret_cast<uint16_t *>(a.vcache)[(long)pos * kvw + kvh * hd + i] =
          float_to_half_bits(vc[i]);
    }
  }
  csync();
  if (tr) tr[2] = global_timer_ns();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const float4 q0 = reinterpret_cast<const float4 *>(q)[lane * 2];
  const float4 q1 = reinterpret_cast<const float4 *>(q)[lane * 2 + 1];
  uint64_t *sc = a.sc + (long)h * a.ctx;
  // scores of the share: two K jobs at a time, warp per position, lane owns 8 dims
  for (int g0 = 0; g0 < nk; g0 += 2) {
    const int g1 = min(g0 + 1, nk - 1);
    cp_async_wait_pending(ng - 1 - g1);
    csync();
    if (tr && g0 == 0) tr[14] = global_timer_ns();
    const int p0 = lo + g0 * kFKChunk, count = min((g1 - g0 + 1) * kFKChunk, hi - p0);
    for (int pp = warp; pp < count; pp += 2 * kFWarps) {
      const bool two = pp + kFWarps < count;
      auto row = [&](int x) {
        return slots + (size_t)((g0 + x / kFKChunk) % kFAttnSlots) * kFAttnSlot +
               (size_t)(x % kFKChunk) * rb;
      };
      double s0 = key_partial_staged(row(pp), hd, a.q8, q0, q1, lane);
      double s1 = two ? key_partial_staged(row(pp + kFWarps), hd, a.q8, q0, q1, lane) : 0.0;
      warp_sum2_f64(s0, s1);
      if (lane == 0) {
        const float v0 = __fmul_rn((float)s0, scale);
        pr[p0 + pp] = v0;
        st_word(sc + p0 + pp, tagged(v0, tag));
        if (two) {
          const float v1 = __fmul_rn((float)s1, scale);
          pr[p0 + pp + kFWarps] = v1;
          st_word(sc + p0 + pp + kFWarps, tagged(v1, tag));
        }
      }
    }
    csync();  // the slots are free again
    if (tr && g0 == 0) tr[15] = global_timer_ns();
    for (int g = g0; g <= g1; ++g) refill(g);
  }
  if (tr) tr[3] = global_timer_ns();
  // the current position's score (every CTA of the head computes it)
  float s_cur;
  {
    const double s = fsum_f64(i < hd ? (double)__fmul_rn(q[i], kc[i]) : 0.0, red);
    s_cur = __fmul_rn((float)s, scale);
  }
  // every share's scores: the other CTAs' from their tagged words
  {
    float v[kFAttnMaxPos / kFThreads];
    const int cnt = i < pos ? (pos - i + kFThreads - 1) / kFThreads : 0;
    ok = wait_words<kFAttnMaxPos / kFThreads>(sc, i, kFThreads, cnt, tag, v, c);
#pragma unroll
    for (int j = 0; j < kFAttnMaxPos / kFThreads; ++j)
      if (j < cnt) pr[i + j * kFThreads] = v[j];
    if (!csync_and(ok)) return false;
  }
  if (tr) tr[4] = global_timer_ns();
  float m = -INFINITY;
  for (int p = i; p < pos; p += kFThreads) m = fmaxf(m, pr[p]);
  const float M = fmaxf(s_cur, fmax_f32(m, fred));
  if (tr) tr[10] = global_timer_ns();
  for (int p = i; p < pos; p += kFThreads) pr[p] = exp_cr(__fsub_rn(pr[p], M));
  csync();
  if (tr) tr[11] = global_timer_ns();
  // share r's total: thread j < kAttnThreads of attention_decode_kernel sums
  // positions j, j + kAttnThreads, ... of the share; warps in butterflies;
  // the eight warps in order
  // (a warp past the share's positions sums zeros: its tree is +0.0)
  {
    const int wn = min(kAttnThreads / 32, (per + 31) / 32);  // warps with positions
    for (int t = warp; t < 8 * wn; t += kFWarps) {
      const int r = t / wn, w = t % wn;
      const int lo_r = min(pos, r * per), n_r = min(pos, lo_r + per) - lo_r;
      double y = 0.0;
      for (int pp = w * 32 + lane; pp < n_r; pp += kAttnThreads) y += (double)pr[lo_r + pp];
      y = warp_sum_f64(y);
      if (lane == 0) tw[r * (kAttnThreads / 32) + w] = y;
    }
    if (i < 64 && (i & 7) >= wn) tw[i] = 0.0;
  }
  csync();
  if (tr) tr[12] = global_timer_ns();
  if (i < 8) {
    double t = 0.0;
    for (int w = 0; w < kAttnThreads / 32; ++w) t += tw[i * 8 + w];
    tot[i] = t;
  }
  csync();
  if (tr) tr[13] = global_timer_ns();
  double total = 0.0;
  for (int r = 0; r < kAttnSplit; ++r) total += tot[r];
  const float e_cur = exp_cr(__fsub_rn(s_cur, M));
  total += (double)e_cur;
  const float inv = (float)(1.0 / total);
  if (!is_finite_f(M) && i == 0 && rank == 0) report(c.status, kStatusNonfinite);
  const float p_cur = round_f16(__fmul_rn(e_cur, inv));
  for (int p = i; p < pos; p += kFThreads) pr[p] = round_f16(__fmul_rn(pr[p], inv));
  if (tr) tr[8] = global_timer_ns();
  // values: thread (share r, dimension dl) sums the share's positions in order
  const int vr = i >> 5, dl = i & 31;
  const int vlo = min(pos, vr * per), vhi = min(pos, vlo + per);
  double acc = -0.0;
  for (int k0 = 0; k0 < nv; k0 += 2) {
    const int k1 = min(k0 + 1, nv - 1);
    cp_async_wait_pending(ng - 1 - (nk + k1));
    csync();
    if (i < kAttnThreads) {
      for (int k = k0; k <= k1; ++k) {
        const uint8_t *vb = slots + (size_t)((nk + k) % kFAttnSlots) * kFAttnSlot;
        const int p0 = vlo + k * kFVDepth, count = min(kFVDepth, vhi - p0);
        if (a.q8) {
          const uint32_t *sw = reinterpret_cast<const uint32_t *>(vb + 8 * kFVDepth * 32);
          for (int t = 0; t < count; ++t) {
            const int slot = vr * kFVDepth + t;
            const uint32_t word = sw[slot];
            const float d = half_bits_to_float((uint16_t)(rank & 1 ? word >> 16 : word));
            const float v = __fmul_rn(d, (float)(int8_t)vb[slot * 32 + dl]);
            acc += (double)__fmul_rn(pr[p0 + t], v);
          }
        } else {
          for (int t = 0; t < count; ++t) {
            const int slot = vr * kFVDepth + t;
            const float v =
                half_bits_to_float(reinterpret_cast<const uint16_t *>(vb + slot * 64)[dl]);
            acc += (double)__fmul_rn(pr[p0 + t], v);
          }
        }
      }
    }
    csync();  // the slots are free again
    for (int k = k0; k <= k1; ++k) refill(nk + k);
  }
  if (i < kAttnThreads) part[vr * 32 + dl] = acc;
  csync();
  if (tr) tr[9] = global_timer_ns();
  // this CTA's output dimensions: the shares in rank order, the current
  // position, the gate
  if (i < dims) {
    const int d = rank * dims + i;
    double sum = -0.0;
    for (int r = 0; r < kAttnSplit; ++r) sum += part[r * 32 + i];
    const float out = (float)(sum + (double)__fmul_rn(p_cur, vc[d]));
    st_word(a.out + (long)h * hd + d, tagged(__fmul_rn(out, sigmoid_f(gs[i])), tag));
  }
  return true;
}

// ---- the kernel --------------------------------------------------------------------

template <int KIND>
__global__ void __launch_bounds__(kFBlock, 1) decode_flow_kernel(FlowArgs fa) {
  extern __shared__ __align__(128) uint8_t smem[];
  FRing rg;
  rg.data = smem;
  rg.bar = reinterpret_cast<uint64_t *>(smem + kFOffBars);
  uint64_t *dbar = rg.bar + kFSlots;  // [kFDescBufs] descriptor arrivals
  rg.off = reinterpret_cast<uint32_t *>(smem + kFOffMeta);
  rg.len = rg.off + kFSlots;
  rg.tail = rg.len + kFSlots;
  rg.released = rg.tail + 1;
  rg.issued = rg.tail + 2;
  rg.issued_live = rg.tail + 3;
  rg.desc_done = rg.tail + 8;
  rg.desc_fetched = rg.tail + 9;
  rg.issue_ts = reinterpret_cast<unsigned long long *>(smem + kFOffIssue);
  const int tid = threadIdx.x;
  if (tid < kFSlots + kFDescBufs) mbar_init(&rg.bar[tid], 1);
  if (tid < 16) rg.tail[tid] = 0u;
  mbar_init_fence();
  __syncthreads();
  FlowCtl c;
  c.status = fa.status;
  c.abort = fa.sync + 1;
  const int pos = *fa.st.position;
  const uint32_t ep = fa.sync[2];
  bool ok = true;
  constexpr int D = kFDescBufs;
  if (tid >= kFThreads) {
    if (tid == kFThreads) {
      // lane 0 of the streaming warp: the weight stream
      flow_producer<KIND>(fa, rg, c);
    } else if (tid == kFThreads + 1) {
      // lane 1: phase descriptors into D buffers; descriptor q goes into
      // buffer q % D once the compute warps finished phase q - D
      Spin sp;
      for (int q = 0; q < fa.nphases; ++q) {
        bool room = true;
        while (q >= D && (int)ld_acquire_cta(rg.desc_done) < q - D + 1) {
          if (!sp.again(c)) {
            room = false;
            break;
          }
          __nanosleep(32);
        }
        if (!room) break;
        fence_proxy_async_smem();  // the buffer was read through the generic proxy
        mbar_arrive_expect_tx(&dbar[q % D], (unsigned)sizeof(FPhase));
        bulk_g2s(smem + kFOffDesc + (q % D) * kFDescBytes, fa.phases + q, (unsigned)sizeof(FPhase),
                 &dbar[q % D]);
        st_release_cta(rg.desc_fetched, (uint32_t)(q + 1));
      }
    }
  } else {
    // the compute warps: descriptor p arrives in buffer p % D
    int cons = 0, waited = 0;
    // descriptor p + 1 is awaited (thread 511) inside phase p's closing barrier
    ok = csync_and(tid != kFThreads - 1 || mbar_wait_bounded(&dbar[0], 0u, c.status));
    if (!ok && tid == 0) flow_raise(c);
    for (int p = 0; p < fa.nphases && ok; ++p) {
      unsigned long long *tr = fa.trace && blockIdx.x == 0 && tid == 0 ? fa.trace + 16 * p : nullptr;
      if (tr) tr[5] = tr[0] = global_timer_ns();
      waited = p + 1;
      const FPhase &ph = *reinterpret_cast<const FPhase *>(smem + kFOffDesc + (p % D) * kFDescBytes);
      if (tr) tr[6] = global_timer_ns();
      const uint32_t tag = flow_tag(ep, ph.k);
      switch (ph.type) {
        case kFEmbed:
          flow_embed<KIND>(ph.em, fa.st, pos, tag, c.status);
          break;
        case kFProj:
          ok = flow_proj<KIND>(ph.pr, rg, smem, ep, tag, cons, c, tr,
                               fa.trace_cta ? fa.trace_cta + ((size_t)p * gridDim.x + blockIdx.x) * 4
                                            : nullptr,
                               fa.trace && blockIdx.x == 0 ? fa.trace + 16 * p : nullptr);
          break;
        case kFGdn:
          ok = flow_gdn(ph.gd, pos, smem, ep, tag, c);
          break;
        default:
          ok = flow_attn(ph.at, pos, smem, ep, tag, c, tr);
          break;
      }
      const bool next = tid != kFThreads - 1 || p + 1 >= fa.nphases ||
                        mbar_wait_bounded(&dbar[(p + 1) % D], (unsigned)((p + 1) / D) & 1u,
                                          c.status);
      ok = csync_and(ok && next);
      if (!ok && tid == 0) flow_raise(c);
      if (tid == 0) st_release_cta(rg.desc_done, (uint32_t)(p + 1));  // buffer p % D is free
      if (tr) tr[7] = global_timer_ns();
      if (fa.trace_cta && tid == 0)
        fa.trace_cta[((size_t)p * gridDim.x + blockIdx.x) * 4 + 2] = global_timer_ns();
    }
    if (!ok && tid == 0) st_release_cta(rg.tail + 10, (uint32_t)waited);
  }
  cp_async_wait_all();  // an aborted phase may leave a residual copy in flight
  __syncthreads();
  if (tid == 0 && !ok) {
    // aborted: descriptor copies may still be in flight
    const uint32_t fetched = *rg.desc_fetched, waited = rg.tail[10];
    for (uint32_t q = waited; q < fetched; ++q)
      mbar_wait_bounded(&dbar[q % D], (q / D) & 1u, c.status);
  }
  if (tid == 0) {
    // every piece the producer issued was consumed, or is drained here
    const uint32_t issued = *rg.issued, released = *rg.released;
    for (uint32_t i = released; i < issued; ++i)
      mbar_wait_bounded(&rg.bar[i % kFSlots], (i / kFSlots) & 1u, fa.status);
    // the last CTA to finish advances the step
    if (ok && !flow_aborted(c)) {
      __threadfence();
      const unsigned done = atomicAdd(&fa.sync[0], 1u);
      if (done == gridDim.x - 1) {
        __threadfence();
        const int next = pos + 1;
        // publish the step's greedy key and clear the working one
        const unsigned long long k = *reinterpret_cast<volatile unsigned long long *>(fa.key);
        *fa.st.argmax = k;
        *fa.key = 0ull;
        if (fa.write_greedy && next >= *fa.st.prompt_end)
          fa.st.tokens[next] = 0xffffffffu - (unsigned)(k & 0xffffffffull);
        *fa.st.position = next;
        fa.sync[2] = ep + 1u;
        fa.sync[0] = 0u;
        __threadfence();
      }
    }
  }
}

}  // namespace prism
