// persist.cuh -- the Qwen3.5-style decode step as ONE persistent kernel.
//
// One cooperative launch per token, one CTA per SM, 512 threads.  The step
// is a host-built list of phases (embedding, projection groups, Gated
// DeltaNet, attention); consecutive phases are separated by a grid barrier.
// What makes it fast is that the weights never wait for the barriers:
// thread 0 of every CTA walks the phase list ahead of the computation and
// streams the weight tiles this CTA will consume (tile t of a projection
// goes to CTA t mod grid) into a 160 KB shared-memory ring with bulk copies,
// across phase boundaries.  A projection phase then only stages its Q8_K
// activation and runs the integer dots on tiles that are (usually) already
// resident, so a step costs about one barrier plus a short compute per
// phase, while HBM streams the next phases' weights underneath.
//
// The arithmetic is that of the per-kernel path (matvec.cuh,
// model_kernels.cuh): the same unit dots, binary32 chains, binary64
// reductions in the same order, the same transcendentals, so both paths give
// identical bits.  The attention's cluster exchange (distributed shared
// memory) becomes an exchange through global memory between the eight CTAs
// of a head, ordered by per-head arrival counters.
//
// Every wait is bounded (kWaitLimitNs): a CTA that gives up raises the
// step's abort word and the timeout status; the others stop at their next
// wait.  Barrier counters are zeroed by the CTA that finishes the step last.
#pragma once

#include "common.cuh"
#include "matvec.cuh"
#include "model_kernels.cuh"

namespace prism {

constexpr int kPThreads = 512;
constexpr int kPWarps = kPThreads / 32;
constexpr int kRingBytes = 160 * 1024;
constexpr int kRingSlots = 32;
constexpr int kGdnSlices = 8;  // CTAs per value head: 16 state rows each
constexpr int kPMaxScores = 2048;
// shared-memory layout
constexpr int kPActBytes = 19456;                  // MatvecSmem activation area, nb <= 64
constexpr int kPTermsBytes = 2 * kMaxNb * 32 * 4;  // terms [upt][h]
constexpr int kPScratchBytes = 24576;  // attention: 8 KB + kPMaxScores scores
constexpr int kPOffAct = kRingBytes;
constexpr int kPOffTerms = kPOffAct + kPActBytes;
constexpr int kPOffScratch = kPOffTerms + kPTermsBytes;
constexpr int kPOffMeta = kPOffScratch + kPScratchBytes;  // bars, ring offsets/lengths, flags
// terms + scratch form one contiguous work area, used to stage a phase's
// inputs before the terms are written
constexpr int kPWorkBytes = kPTermsBytes + kPScratchBytes;
constexpr int kPOffPlan = kPOffMeta + kRingSlots * 16 + 64;  // the producer's phase plan
constexpr int kPOffPhase = kPOffPlan + 128;                 // phase descriptors, double-buffered
constexpr int kPPhaseBytes = 1024;
constexpr int kPSmemBytes = kPOffPhase + 2 * kPPhaseBytes;

enum PhaseType : int { kPhEmbed = 0, kPhMatvec = 1, kPhGdn = 2, kPhAttn = 3 };
enum PPrologue : int { kPPRms = 0, kPPF32 = 1, kPPGated = 2 };

struct PMatvec {
  MvWeight w[kMaxGroup];
  int count, nb, epi, prologue;
  int tile_start[kMaxGroup + 1];
  int ntiles;                 // tiles of the phase (the pair: per weight)
  const float *in;            // f32 activation
  const float *norm_w;        // Rms: [nb*256]; Gated: [head_dim]
  const float *zgate;         // Gated: [heads*head_dim]
  float *gated_out;           // Gated: CTA 0 also stores the gated vector here
  int heads, head_dim;
  float eps;
  unsigned long long *argmax_key;
};

struct PAttn {
  AttnArgs a;
  float *smax;      // [heads][kAttnSplit]
  double *stot;     // [heads][kAttnSplit]
  double *part;     // [heads][kAttnSplit][hd]
  unsigned *hsync;  // [heads] arrival counters
};

struct PEmbed {
  const uint8_t *units;
  int h, nb, vocab, n;
  float *hidden;
};

struct alignas(16) Phase {
  int type;
  PMatvec mv;
  GdnArgs gdn;
  PAttn at;
  PEmbed em;
};

static_assert(sizeof(Phase) <= kPPhaseBytes && sizeof(Phase) % 16 == 0, "phase descriptor");

// Weight streaming plan of one phase: what the producer needs to issue its
// tiles (no tiles for phases other than projections).
struct PTiles {
  const uint8_t *units[kMaxGroup];
  int tile_start[kMaxGroup + 1];
  int part[kMaxGroup];  // bytes of one tile of weight g (nb units)
  int ntiles, count, pair;
};
static_assert(sizeof(PTiles) <= 128, "plan");

struct PersistArgs {
  const Phase *phases;
  const PTiles *tiles;  // [nphases]
  int nphases;
  StepState st;
  int write_greedy;
  unsigned *sync;       // [0] grid arrivals, [1] finished CTAs, [2] abort
  unsigned *hsync;      // all attention arrival counters (zeroed at step end)
  int nhsync;
  unsigned *status;
  // optional, CTA 0's timeline: 8 slots per phase -- [0] start (after the
  // barrier) and [7] end (arrival at the next barrier) in globaltimer ns;
  // [5] start, [1] inputs staged, [2] first tiles resident, [3] their dots
  // done, [4] their chains done in SM clock cycles (projections only)
  unsigned long long *trace;
};

// ---- synchronisation -------------------------------------------------------

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Weight streaming state of a CTA; only thread 0 uses it.
struct Producer {
  int p, t;              // next (phase, tile) to issue
  uint32_t head, tail;   // ring bytes issued / released (monotonic)
  int issued, consumed;  // tiles
};

struct RingMeta {
  uint64_t *bar;   // [kRingSlots]
  uint32_t *off;   // [kRingSlots] data offset in the ring
  uint32_t *len;   // [kRingSlots] bytes to release (padding + data)
  int *flag;       // CTA-wide result of thread 0's waits
  PTiles *plan;    // the producer's current phase plan
};

// Issue as many of this CTA's upcoming tiles as the ring has room for.  The
// current phase's plan is cached in shared memory; the next one is read
// from global memory only when the cursor moves to it.
template <int KIND>
__device__ void pump(Producer &pr, const PersistArgs &pa, uint8_t *ring, const RingMeta &rm) {
  PTiles *plan = rm.plan;
  bool fenced = false;
  for (;;) {
    if (pr.t >= plan->ntiles) {
      if (++pr.p >= pa.nphases) {
        plan->ntiles = 0;
        pr.p = pa.nphases;
        return;
      }
      *plan = pa.tiles[pr.p];
      pr.t = blockIdx.x;
      continue;
    }
    if (pr.issued - pr.consumed >= kRingSlots) return;
    int g = 0;
    if (!plan->pair)
      for (int i = 1; i < plan->count; ++i)
        if (pr.t >= plan->tile_start[i]) g = i;
    const uint32_t part = (uint32_t)plan->part[g];
    const uint32_t bytes = plan->pair ? 2 * part : part;
    uint32_t off = pr.head % kRingBytes;
    const uint32_t pad = off + bytes > (uint32_t)kRingBytes ? kRingBytes - off : 0u;
    if (pr.head + pad + bytes - pr.tail > (uint32_t)kRingBytes) return;
    if (!fenced) {
      fence_proxy_async_smem();  // released space was read through the generic proxy
      fenced = true;
    }
    pr.head += pad;
    off = pr.head % kRingBytes;
    const int slot = pr.issued % kRingSlots;
    rm.off[slot] = off;
    rm.len[slot] = pad + bytes;
    const int lt = plan->pair ? pr.t : pr.t - plan->tile_start[g];
    mbar_arrive_expect_tx(&rm.bar[slot], bytes);
    bulk_g2s(ring + off, plan->units[g] + (size_t)lt * part, part, &rm.bar[slot]);
    if (plan->pair)
      bulk_g2s(ring + off + part, plan->units[1] + (size_t)lt * part, part, &rm.bar[slot]);
    pr.head += bytes;
    ++pr.issued;
    pr.t += gridDim.x;
  }
}

__device__ __forceinline__ bool aborted(const PersistArgs &pa) {
  return *reinterpret_cast<volatile const unsigned *>(&pa.sync[2]) != 0u;
}

__device__ __forceinline__ void raise_abort(const PersistArgs &pa) {
  report(pa.status, kStatusTimeout);
  atomicExch(&pa.sync[2], 1u);
}

// Grid-wide barrier number `k` of the step (arrivals are cumulative).  Thread
// 0 keeps streaming weights while it waits.  Returns false on abort.
template <int KIND>
__device__ bool grid_barrier(const PersistArgs &pa, unsigned k, Producer &pr, uint8_t *ring,
                             const RingMeta &rm) {
  __syncthreads();
  if (pa.trace && blockIdx.x == 0 && threadIdx.x == 0) pa.trace[8 * (k - 1) + 7] = global_timer_ns();
  if (threadIdx.x == 0) {
    int ok = 1;
    // release: this CTA's writes (ordered by the bar.sync above) before the arrival
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&pa.sync[0]) : "memory");
    const unsigned target = k * gridDim.x;
    const unsigned long long t0 = global_timer_ns();
    while (ld_acquire_gpu(&pa.sync[0]) < target) {
      pump<KIND>(pr, pa, ring, rm);
      if (aborted(pa)) {
        ok = 0;
        break;
      }
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        raise_abort(pa);
        ok = 0;
        break;
      }
    }
    *rm.flag = ok;
  }
  __syncthreads();
  return *rm.flag != 0;
}

// Arrival `k` of the kAttnSplit CTAs of one attention head.
__device__ bool head_barrier(const PersistArgs &pa, unsigned *counter, unsigned k, int *flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(counter, 1u);
    const unsigned target = k * kAttnSplit;
    const unsigned long long t0 = global_timer_ns();
    while (ld_acquire_gpu(counter) < target) {
      if (aborted(pa)) {
        ok = 0;
        break;
      }
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        raise_abort(pa);
        ok = 0;
        break;
      }
    }
    __threadfence();
    *flag = ok;
  }
  __syncthreads();
  return *flag != 0;
}

// ---- phases ------------------------------------------------------------------

// Gated output norm of the GDN heads (the tail of gdn_decode_kernel):
// y = RMSNorm(o_h) * w * SiLU(z), one warp per head, the binary64 sum of
// squares in the same order as the 512-thread block sum of that kernel.
// o, z, w are shared-memory copies.
__device__ void gated_heads(const PMatvec &mv, const float *o_all, const float *z_all,
                            const float *w, float *out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = mv.head_dim;  // 128
  for (int h = warp; h < mv.heads; h += kPWarps) {
    const float *o = o_all + h * S;
    double t = 0.0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float v = o[32 * q + lane];
      t += warp_sum_f64((double)__fmul_rn(v, v));
    }
    const float mean = (float)(t / (double)S);
    const float nscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, mv.eps)));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = 32 * q + lane;
      const float normed = __fmul_rn(__fmul_rn(o[i], nscale), w[i]);
      const float y = __fmul_rn(normed, silu_f(z_all[h * S + i]));
      out[h * S + i] = y;
      if (blockIdx.x == 0 && mv.gated_out) mv.gated_out[h * S + i] = y;
    }
  }
}

// Copy n floats (n % 4 == 0) from global to shared memory, all threads.
__device__ __forceinline__ void load_f32(float *dst, const float *src, int n) {
  for (int i = threadIdx.x * 4; i < n; i += kPThreads * 4)
    *reinterpret_cast<float4 *>(dst + i) = *reinterpret_cast<const float4 *>(src + i);
}

// Two units of one tile height at once: independent work for the scheduler
// to interleave (each unit's dot is a short dependent chain).
template <int KIND, int H>
__device__ __forceinline__ void unit_pair(const uint8_t *ua, const int8_t *ava, int asa,
                                          const int16_t *gsa, float sa_, float *outa,
                                          const uint8_t *ub, const int8_t *avb, int asb,
                                          const int16_t *gsb, float sb_, float *outb,
                                          int lane) {
  int da, db, d2a, d2b;
  float ta, tb;
  unit_terms<KIND, H>(ua, ava, asa, gsa, sa_, lane, da, d2a, ta);
  unit_terms<KIND, H>(ub, avb, asb, gsb, sb_, lane, db, d2b, tb);
  if (lane < H) {
    outa[lane % H] = ta;
    outb[lane % H] = tb;
  }
}

template <int KIND>
__device__ __forceinline__ void unit_dispatch(int H, const uint8_t *unit, const int8_t *av,
                                              int asum, const int16_t *gs, float s, int lane,
                                              float *out) {
  int dot, dot2;
  float term;
  if (H == 32)
    unit_terms<KIND, 32>(unit, av, asum, gs, s, lane, dot, dot2, term);
  else if (H == 16)
    unit_terms<KIND, 16>(unit, av, asum, gs, s, lane, dot, dot2, term);
  else
    unit_terms<KIND, 8>(unit, av, asum, gs, s, lane, dot, dot2, term);
  if (lane < H) out[lane % H] = term;
}

// A projection phase: stage the Q8_K activation once, then take this CTA's
// tiles (t = blockIdx.x + k * grid) in batches that the ring and the term
// buffer hold together -- all units of a batch are spread over the 16 warps,
// then every row's chain runs at once (one thread per row).
template <int KIND>
__device__ bool run_matvec(const PMatvec &mv, const PersistArgs &pa, uint8_t *smem,
                           Producer &pr, const RingMeta &rm, int &cons, int phase) {
  unsigned long long *tr =
      pa.trace && blockIdx.x == 0 && threadIdx.x == 0 ? pa.trace + 8 * phase : nullptr;
  const int T = mv.ntiles, G = gridDim.x;
  if ((int)blockIdx.x >= T) return true;
  const bool pair = mv.epi == kEpiSwiglu;
  const int nb = mv.nb, upt = pair ? 2 * nb : nb;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t *act = smem + kPOffAct;
  float *terms = reinterpret_cast<float *>(smem + kPOffTerms);
  float *work = terms;  // [kPWorkBytes]: staged inputs, then terms
  const MatvecSmem L(nb, 32, unit_bytes(KIND, 32), upt);
  MvArgs sa;
  sa.nb = nb;
  sa.eps = mv.eps;
  sa.norm_w = mv.norm_w;
  sa.status = pa.status;
  sa.pinned = 0;
  sa.prologue = mv.prologue == kPPRms ? kProRmsNorm : kProF32;
  sa.in0 = mv.in;
  const int n = nb * 256;
  // stage the inputs into shared memory with all loads in flight at once
  if (mv.prologue == kPPGated) {
    const int S = mv.head_dim;
    float *o = work, *z = work + n, *w = work + 2 * n, *y = work + 2 * n + S;
    if ((3 * n + S) * 4 <= kPWorkBytes) {
      load_f32(o, mv.in, n);
      load_f32(z, mv.zgate, n);
      load_f32(w, mv.norm_w, S);
      __syncthreads();
      gated_heads(mv, o, z, w, y);
      __syncthreads();
      sa.in0 = y;
    }
  } else if (mv.prologue == kPPRms && 2 * n * 4 <= kPWorkBytes) {
    load_f32(work, mv.in, n);
    load_f32(work + n, mv.norm_w, n);
    __syncthreads();
    sa.in0 = work;
    sa.norm_w = work + n;
  } else if (mv.prologue == kPPF32 && n * 4 <= kPWorkBytes) {
    load_f32(work, mv.in, n);
    __syncthreads();
    sa.in0 = work;
  }
  stage_from_f32(sa, L, act);
  __syncthreads();
  if (tr) tr[1] = clock64();
  const int8_t *values = reinterpret_cast<const int8_t *>(act + L.act_values());
  const float *ascale = reinterpret_cast<const float *>(act + L.act_scale());
  const int16_t *asums = reinterpret_cast<const int16_t *>(act + L.act_sums());
  const int *aasum = reinterpret_cast<const int *>(act + L.act_asum());
  int maxtile = 0;
  for (int g = 0; g < mv.count; ++g)
    maxtile = max(maxtile, nb * unit_bytes(KIND, mv.w[g].h) * (pair ? 2 : 1));
  // All of this CTA's tiles in one batch when the ring holds them together
  // (they were streamed during earlier phases); otherwise batches of half
  // the ring, so that one batch computes while the next one streams in.
  const int mine = (T - (int)blockIdx.x + G - 1) / G;
  const int fit = kRingBytes / maxtile - 1;  // one tile's worth lost to wrap padding
  int cap = min(kPWarps, (kPTermsBytes / 4) / (upt * 32));
  cap = mine <= min(cap, fit) ? mine : min(cap, max(1, fit / 2));
  auto group_of_tile = [&](int t) {
    int g = 0;
    if (!pair)
      for (int i = 1; i < mv.count; ++i)
        if (t >= mv.tile_start[i]) g = i;
    return g;
  };
  unsigned long long best = 0ull;
  for (int k0 = 0; k0 < mine; k0 += cap) {
    const int B = min(cap, mine - k0);
    // the chain thread of this batch (warp = tile, lane = row) loads its
    // residual now, so the load overlaps the dot products
    const int ck = warp, ct = blockIdx.x + (k0 + ck) * G;
    const int cg = ck < B ? group_of_tile(ct) : 0;
    const MvWeight &cw = mv.w[cg];
    const int corow = (pair ? ct : ct - mv.tile_start[cg]) * cw.h + lane;
    const bool chain = ck < B && lane < cw.h;
    if (tid == 0 && pr.issued < cons + B) pump<KIND>(pr, pa, smem, rm);
    if (tr && k0 == 0) tr[6] = clock64();
    bool arrived = true;
    for (int k = 0; k < B && arrived; ++k)
      arrived = mbar_wait_bounded(&rm.bar[(cons + k) % kRingSlots],
                                  (unsigned)((cons + k) / kRingSlots) & 1u, pa.status);
    if (!__syncthreads_and(arrived)) {
      if (tid == 0) raise_abort(pa);
      return false;
    }
    if (tr && k0 == 0) tr[2] = clock64();
    const int total = B * upt;
    for (int u = warp; u < total; u += 2 * kPWarps) {
      const int u2 = u + kPWarps;
      const int k = u / upt, j = u - k * upt;
      const int g = group_of_tile(blockIdx.x + (k0 + k) * G);
      const int H = mv.w[g].h;
      const uint8_t *data = smem + rm.off[(cons + k) % kRingSlots];
      const int b = pair && j >= nb ? j - nb : j;
      const uint8_t *ua = data + j * unit_bytes(KIND, H);
      float *oa = terms + k * upt * 32 + j * H;
      int H2 = -1, b2 = 0;
      const uint8_t *ub = nullptr;
      float *ob = nullptr;
      if (u2 < total) {
        const int k2 = u2 / upt, j2 = u2 - k2 * upt;
        const int g2 = group_of_tile(blockIdx.x + (k0 + k2) * G);
        H2 = mv.w[g2].h;
        b2 = pair && j2 >= nb ? j2 - nb : j2;
        ub = smem + rm.off[(cons + k2) % kRingSlots] + j2 * unit_bytes(KIND, H2);
        ob = terms + k2 * upt * 32 + j2 * H2;
      }
      if (H2 == H) {
        if (H == 32)
          unit_pair<KIND, 32>(ua, values + b * 256, aasum[b], asums + b * 16, ascale[b], oa, ub,
                              values + b2 * 256, aasum[b2], asums + b2 * 16, ascale[b2], ob, lane);
        else if (H == 16)
          unit_pair<KIND, 16>(ua, values + b * 256, aasum[b], asums + b * 16, ascale[b], oa, ub,
                              values + b2 * 256, aasum[b2], asums + b2 * 16, ascale[b2], ob, lane);
        else
          unit_pair<KIND, 8>(ua, values + b * 256, aasum[b], asums + b * 16, ascale[b], oa, ub,
                             values + b2 * 256, aasum[b2], asums + b2 * 16, ascale[b2], ob, lane);
      } else {
        unit_dispatch<KIND>(H, ua, values + b * 256, aasum[b], asums + b * 16, ascale[b], lane,
                            oa);
        if (H2 > 0)
          unit_dispatch<KIND>(H2, ub, values + b2 * 256, aasum[b2], asums + b2 * 16, ascale[b2],
                              lane, ob);
      }
    }
    __syncthreads();
    if (tr && k0 == 0) tr[3] = clock64();
    if (chain) {
      const int H = cw.h, r = lane;
      const float *tk = terms + ck * upt * 32;
      // the reference's chain: sum = 0; sum += term_b for b in order
      float sum = 0.0f;
      for (int b = 0; b < nb; ++b) sum = __fadd_rn(sum, tk[b * H + r]);
      if (pair) {
        float gsum = 0.0f;
        for (int b = nb; b < 2 * nb; ++b) gsum = __fadd_rn(gsum, tk[b * H + r]);
        if (corow < cw.rows) {
          const float hv = __fmul_rn(sum, silu_f(gsum));
          if (!is_finite_f(sum) || !is_finite_f(gsum)) report(pa.status, kStatusNonfinite);
          cw.y[corow] = hv;
        }
      } else if (corow < cw.rows) {
        if (cw.residual) sum = __fadd_rn(cw.residual[corow], sum);
        if (!is_finite_f(sum)) report(pa.status, kStatusNonfinite);
        if (cw.y) cw.y[corow] = sum;
        if (mv.epi == kEpiArgmax) {
          const unsigned long long key = argmax_key(sum, corow);
          best = key > best ? key : best;
        }
      }
    }
    __syncthreads();  // the batch's ring space is free again
    if (tr && k0 == 0) tr[4] = clock64();
    if (tid == 0) {
      for (int k = 0; k < B; ++k) pr.tail += rm.len[(cons + k) % kRingSlots];
      pr.consumed += B;
      // more batches: stream the next one now; otherwise the barrier's
      // wait loop streams the following phases
      if (k0 + cap < mine) pump<KIND>(pr, pa, smem, rm);
    }
    cons += B;
  }
  if (mv.epi == kEpiArgmax) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0 && best) atomicMax(mv.argmax_key, best);
  }
  return true;
}

// Gated DeltaNet layer, value head h split over kGdnSlices CTAs of 16 state
// rows (arithmetic of gdn_decode_kernel; the output norm runs in the next
// projection's prologue).  o (pre-norm) goes to a.attended.
__device__ void run_gdn(const GdnArgs &a, int pos, uint8_t *scratch,
                        const float4 *preloaded = nullptr) {
  constexpr int S = 128, R = S / kGdnSlices;
  if ((int)blockIdx.x >= a.values * kGdnSlices) return;
  float *q = reinterpret_cast<float *>(scratch);  // [S]
  float *k = q + S;                              // [S]
  float *v = k + S;                              // [R]
  double *red = reinterpret_cast<double *>(v + R + 16);
  float *sdb = reinterpret_cast<float *>(red + kPWarps);  // decay, beta
  const int h = blockIdx.x / kGdnSlices, slice = blockIdx.x % kGdnSlices, r0 = slice * R;
  const int kh = h % a.groups, kw = a.groups * S, hist = a.conv_k - 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int parity = pos & 1;
  const float *hist_in = a.conv_state + parity * a.conv_buf_stride;
  float *hist_out = a.conv_state + (parity ^ 1) * a.conv_buf_stride;
  // 1. convolution + SiLU of the head's q, k channels and this slice's v
  if (tid < 2 * S + R) {
    const int part = tid < S ? 0 : tid < 2 * S ? 1 : 2;
    const int j = part < 2 ? tid - part * S : r0 + (tid - 2 * S);
    const int ch = part == 0 ? kh * S + j : part == 1 ? kw + kh * S + j : 2 * kw + h * S + j;
    const float projected = a.mixed[ch];
    const float *hj = hist_in + (long)ch * hist;
    const float *cj = a.conv_w + (long)ch * a.conv_k;
    float sum = 0.0f;
    for (int i = 0; i < hist; ++i) sum = __fadd_rn(sum, __fmul_rn(hj[i], cj[i]));
    sum = __fadd_rn(sum, __fmul_rn(projected, cj[hist]));
    const float act = silu_f(sum);
    if (part == 0) q[j] = act;
    else if (part == 1) k[j] = act;
    else v[j - r0] = act;
    if (part == 2 || (h == kh && slice == 0)) {
      float *nj = hist_out + (long)ch * hist;
      for (int i = 0; i + 1 < hist; ++i) nj[i] = hj[i + 1];
      if (hist > 0) nj[hist - 1] = projected;
    }
  }
  if (tid == 0) {
    sdb[0] = recurrent_decay_f(a.alpha_in[h], a.dt_bias[h], a.ssm_a[h], a.status);
    sdb[1] = sigmoid_f(a.beta_in[h]);
  }
  __syncthreads();
  // 2. L2 normalisation of q and k (same block-sum order as the kernel)
  {
    const float xq = tid < S ? q[tid] : 0.0f;
    const float xk = tid < S ? k[tid] : 0.0f;
    const double sq = block_sum_f64(tid < S ? (double)__fmul_rn(xq, xq) : 0.0, red);
    const double sk = block_sum_f64(tid < S ? (double)__fmul_rn(xk, xk) : 0.0, red);
    const float scq = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sq), a.eps));
    const float sck = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sk), a.eps));
    __syncthreads();
    if (tid < S) {
      q[tid] = __fmul_rn(xq, scq);
      k[tid] = __fmul_rn(xk, sck);
    }
  }
  __syncthreads();
  // 3. this slice's state rows, one per warp
  const float decay = sdb[0], beta = sdb[1];
  const float oscale = __fdiv_rn(1.0f, __fsqrt_rn((float)S));
  if (warp < R) {
    const int r = r0 + warp;
    const float4 kk = reinterpret_cast<const float4 *>(k)[lane];
    const float4 qq = reinterpret_cast<const float4 *>(q)[lane];
    float *row = a.state + (long)h * S * S + (long)r * S;
    float4 s = preloaded ? *preloaded : reinterpret_cast<const float4 *>(row)[lane];
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
    if (lane == 0) a.attended[h * S + r] = __fmul_rn((float)dq, oscale);
    if (!__all_sync(0xffffffffu, finite) && lane == 0) report(a.status, kStatusNonfinite);
  }
}

// The kernel-sequence step's Gated DeltaNet layer: value head h split over
// kGdnSlices CTAs of 16 state rows (grid values * kGdnSlices, kPThreads
// threads), run_gdn's arithmetic.  Pre-norm o goes to a.attended; the gated
// output norm runs in the out-projection's prologue (kProGated), for which
// each CTA replaces its 16 z values by SiLU(z) in place.  The state row was
// written by this layer's previous step: it is loaded before the grid
// dependency.
__global__ void __launch_bounds__(kPThreads) gdn_slices_kernel(GdnArgs a) {
  constexpr int S = 128, R = S / kGdnSlices;
  __shared__ __align__(16) uint8_t scratch[2048];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x / kGdnSlices, slice = blockIdx.x % kGdnSlices;
  trace_stamp(a.trace, 0);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (warp < R && h < a.values)
    s = reinterpret_cast<const float4 *>(a.state + (long)h * S * S +
                                         (long)(slice * R + warp) * S)[lane];
  grid_dependency_wait();
  trace_stamp(a.trace, 1);
  grid_dependents_launch();
  run_gdn(a, *a.position, scratch, &s);
  if (threadIdx.x < R && h < a.values) {
    float *z = const_cast<float *>(a.zgate) + (long)h * S + slice * R + threadIdx.x;
    *z = silu_f(*z);
  }
  trace_exit(a.trace);
}

// RMSNorm(x)*w, RoPE, binary16 rounding over hd (== 256) values; threads at
// or past hd take part in the reductions with zeros.
__device__ float p_norm_rope_round(const float *x, const float *w, float eps, int hd, int rope,
                                   const float *cs, float *buf, double *red) {
  const int i = threadIdx.x;
  const float xi = i < hd ? x[i] : 0.0f;
  const double ss = block_sum_f64(i < hd ? (double)__fmul_rn(xi, xi) : 0.0, red);
  const float mean = (float)(ss / (double)hd);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  if (i < hd) buf[i] = __fmul_rn(__fmul_rn(xi, scale), w[i]);
  __syncthreads();
  float out = i < hd ? buf[i] : 0.0f;
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

// Attention for query head h split over kAttnSplit CTAs (arithmetic of
// attention_decode_kernel; hd == 256).
__device__ bool run_attn(const PAttn &pt, const PersistArgs &pa, int pos, uint8_t *scratch,
                         int *flag) {
  const AttnArgs &a = pt.a;
  if ((int)blockIdx.x >= a.heads * kAttnSplit) return true;
  const int hd = a.hd;
  float *q = reinterpret_cast<float *>(scratch);  // [hd]
  float *kc = q + hd;
  float *vc = kc + hd;
  float *buf = vc + hd;
  float *cs = buf + hd;                            // [64]
  double *red = reinterpret_cast<double *>(cs + 64);
  float *fred = reinterpret_cast<float *>(red + kPWarps);
  float *sv = fred + kPWarps;                      // s_cur
  float *scores = reinterpret_cast<float *>(scratch + 8192);
  const int rank = blockIdx.x % kAttnSplit, h = blockIdx.x / kAttnSplit;
  const int group = a.heads / a.kv_heads, kvh = h / group, kvw = a.kv_heads * hd;
  const int i = threadIdx.x, warp = i >> 5, lane = i & 31;
  const int per = (pos + kAttnSplit - 1) / kAttnSplit;
  const int lo = min(pos, rank * per), hi = min(pos, lo + per);
  if (i < a.rope_dim / 2) {
    float theta = (float)pos;
    for (int j = 0; j < i; ++j) theta = __fmul_rn(theta, a.theta_scale);
    const float angle = i < 3 * a.sections[i % 3] ? theta : 0.0f;
    cs[2 * i] = cos_cr(angle);
    cs[2 * i + 1] = sin_cr(angle);
  }
  __syncthreads();
  const float qv = p_norm_rope_round(a.projected + (long)h * 2 * hd, a.q_norm, a.eps, hd,
                                     a.rope_dim, cs, buf, red);
  const float kv_ = p_norm_rope_round(a.key_in + (long)kvh * hd, a.k_norm, a.eps, hd,
                                      a.rope_dim, cs, buf, red);
  if (i < hd) {
    q[i] = qv;
    kc[i] = kv_;
    vc[i] = round_f16(a.value_in[kvh * hd + i]);
    const bool writer = rank == 0 && h % group == 0;
    if (a.q8) {
      const long at = ((long)pos * a.kv_heads + kvh) * q8_0_record_bytes(hd);
      kc[i] = q8_0_roundtrip(kc[i], writer ? reinterpret_cast<uint8_t *>(a.kcache) + at : nullptr,
                             hd, a.status);
      vc[i] = q8_0_roundtrip(vc[i], writer ? reinterpret_cast<uint8_t *>(a.vcache) + at : nullptr,
                             hd, a.status);
    } else if (writer) {
      a.kcache[(long)pos * kvw + kvh * hd + i] = float_to_half_bits(kc[i]);
      a.vcache[(long)pos * kvw + kvh * hd + i] = float_to_half_bits(vc[i]);
    }
  }
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const float4 q0 = reinterpret_cast<const float4 *>(q)[lane * 2];
  const float4 q1 = reinterpret_cast<const float4 *>(q)[lane * 2 + 1];
  for (int p = lo + warp; p < hi; p += kPWarps) {
    const double s = warp_sum_f64(key_partial(a, p, kvh, q0, q1, lane));
    if (lane == 0) scores[p - lo] = __fmul_rn((float)s, scale);
  }
  {
    const double s = block_sum_f64(i < hd ? (double)__fmul_rn(q[i], kc[i]) : 0.0, red);
    if (i == 0) sv[0] = __fmul_rn((float)s, scale);
  }
  __syncthreads();
  const float s_cur = sv[0];
  float m = -INFINITY;
  for (int p = i; p < hi - lo; p += kAttnThreads)
    if (i < kAttnThreads) m = fmaxf(m, scores[p]);
  m = block_max_f32(m, fred);
  if (i == 0) pt.smax[h * kAttnSplit + rank] = m;
  unsigned *ctr = pt.hsync + h;
  if (!head_barrier(pa, ctr, 1, flag)) return false;
  float M = s_cur;
  for (int r = 0; r < kAttnSplit; ++r) M = fmaxf(M, __ldcg(pt.smax + h * kAttnSplit + r));
  double tot = 0.0;
  if (i < kAttnThreads)
    for (int p = i; p < hi - lo; p += kAttnThreads) {
      const float e = exp_cr(__fsub_rn(scores[p], M));
      scores[p] = e;
      tot += (double)e;
    }
  tot = block_sum_f64(tot, red);
  if (i == 0) pt.stot[h * kAttnSplit + rank] = tot;
  if (!head_barrier(pa, ctr, 2, flag)) return false;
  double total = 0.0;
  for (int r = 0; r < kAttnSplit; ++r) total += __ldcg(pt.stot + h * kAttnSplit + r);
  const float e_cur = exp_cr(__fsub_rn(s_cur, M));
  total += (double)e_cur;
  const float inv = (float)(1.0 / total);
  if (!is_finite_f(M) && i == 0 && rank == 0) report(a.status, kStatusNonfinite);
  const float p_cur = round_f16(__fmul_rn(e_cur, inv));
  if (i < kAttnThreads)
    for (int p = i; p < hi - lo; p += kAttnThreads) scores[p] = round_f16(__fmul_rn(scores[p], inv));
  __syncthreads();
  if (i < hd) {
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
    pt.part[((long)h * kAttnSplit + rank) * hd + i] = acc;
  }
  if (!head_barrier(pa, ctr, 3, flag)) return false;
  const int dims = hd / kAttnSplit;
  if (i < dims) {
    const int d = rank * dims + i;
    double sum = -0.0;
    for (int r = 0; r < kAttnSplit; ++r) sum += __ldcg(pt.part + ((long)h * kAttnSplit + r) * hd + d);
    const float out = (float)(sum + (double)__fmul_rn(p_cur, vc[d]));
    const float g = a.projected[(long)(2 * h + 1) * hd + d];
    a.attended[(long)h * hd + d] = __fmul_rn(out, sigmoid_f(g));
  }
  return true;
}

template <int KIND>
__device__ void run_embed(const PEmbed &e, const StepState &st, int pos, unsigned *status) {
  const uint32_t token = st.tokens[pos];
  if (blockIdx.x == 0 && threadIdx.x == 0) *st.argmax = 0ull;
  if (token >= (uint32_t)e.vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(status, kStatusInvalid);
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < e.n; i += gridDim.x * blockDim.x)
    e.hidden[i] = decode_tiled<KIND>(e.units, e.h, e.nb, (int)token, i);
}

// ---- the kernel ----------------------------------------------------------------

template <int KIND>
__global__ void __launch_bounds__(kPThreads, 1) decode_persistent_kernel(PersistArgs pa) {
  extern __shared__ __align__(128) uint8_t smem[];
  RingMeta rm;
  rm.bar = reinterpret_cast<uint64_t *>(smem + kPOffMeta);
  rm.off = reinterpret_cast<uint32_t *>(rm.bar + kRingSlots);
  rm.len = rm.off + kRingSlots;
  rm.flag = reinterpret_cast<int *>(rm.len + kRingSlots);
  rm.plan = reinterpret_cast<PTiles *>(smem + kPOffPlan);
  Phase *cur = reinterpret_cast<Phase *>(smem + kPOffPhase);
  if (threadIdx.x < kRingSlots) mbar_init(&rm.bar[threadIdx.x], 1);
  if (threadIdx.x == 0) rm.plan->ntiles = 0;
  mbar_init_fence();
  __syncthreads();
  const int pos = *pa.st.position;
  Producer pr;
  pr.p = -1;  // the first pump moves to phase 0
  pr.t = 0;
  pr.head = pr.tail = 0;
  pr.issued = pr.consumed = 0;
  if (threadIdx.x == 0) pump<KIND>(pr, pa, smem, rm);
  int cons = 0;
  unsigned barrier = 0;
  bool ok = true;
  // descriptor p is read into buffer p&1 before the barrier that precedes
  // phase p, so its load latency hides behind the barrier
  auto fetch = [&](int p) {
    const uint4 *src = reinterpret_cast<const uint4 *>(pa.phases + p);
    uint4 *dst = reinterpret_cast<uint4 *>(smem + kPOffPhase + (p & 1) * kPPhaseBytes);
    for (int i = threadIdx.x; i < (int)(sizeof(Phase) / 16); i += kPThreads) dst[i] = src[i];
  };
  fetch(0);
  for (int p = 0; p < pa.nphases && ok; ++p) {
    if (p > 0) {
      fetch(p);
      if (!grid_barrier<KIND>(pa, ++barrier, pr, smem, rm)) {
        ok = false;
        break;
      }
    } else {
      __syncthreads();
    }
    if (pa.trace && blockIdx.x == 0 && threadIdx.x == 0) {
      pa.trace[8 * p] = global_timer_ns();
      pa.trace[8 * p + 5] = clock64();
    }
    cur = reinterpret_cast<Phase *>(smem + kPOffPhase + (p & 1) * kPPhaseBytes);
    const Phase *ph = cur;
    switch (ph->type) {
      case kPhEmbed:
        run_embed<KIND>(ph->em, pa.st, pos, pa.status);
        break;
      case kPhMatvec:
        ok = run_matvec<KIND>(ph->mv, pa, smem, pr, rm, cons, p);
        break;
      case kPhGdn:
        run_gdn(ph->gdn, pos, smem + kPOffScratch);
        break;
      default:
        ok = run_attn(ph->at, pa, pos, smem + kPOffScratch, rm.flag);
        break;
    }
  }
  if (!ok && threadIdx.x == 0) {
    // aborted: let this CTA's copies in flight land (bounded) before exiting
    for (int i = pr.consumed; i < pr.issued; ++i)
      mbar_wait_bounded(&rm.bar[i % kRingSlots], (unsigned)(i / kRingSlots) & 1u, pa.status);
  }
  // the last CTA to finish advances the step and clears the counters
  __syncthreads();
  if (pa.trace && blockIdx.x == 0 && threadIdx.x == 0 && ok)
    pa.trace[8 * pa.nphases - 1] = global_timer_ns();
  if (threadIdx.x == 0 && ok) {
    __threadfence();
    const unsigned done = atomicAdd(&pa.sync[1], 1u);
    if (done == gridDim.x - 1) {
      __threadfence();
      const int next = pos + 1;
      if (pa.write_greedy && next >= *pa.st.prompt_end) {
        const unsigned long long key = *reinterpret_cast<volatile unsigned long long *>(pa.st.argmax);
        pa.st.tokens[next] = 0xffffffffu - (unsigned)(key & 0xffffffffull);
      }
      *pa.st.position = next;
      for (int i = 0; i < pa.nhsync; ++i) pa.hsync[i] = 0u;
      pa.sync[0] = 0u;
      pa.sync[1] = 0u;
      __threadfence();
    }
  }
}

}  // namespace prism
