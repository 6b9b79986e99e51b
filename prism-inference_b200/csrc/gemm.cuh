// gemm.cuh -- multi-token packed projection (prefill, batched decode) on the
// 5th-generation tensor cores: tcgen05.mma kind::i8 with TMEM accumulators.
//
// Y[m][n] = sum_b term(m, n, b) over the 256-column blocks b, the reference's
// sequential binary32 chain per output (TQ2_0: src/kernels/tquants.rs:270-287;
// Q2_K: src/kernels/kquants.rs:346-420), here for every token m of a tile
// (the reference's ProjectionTile per-token dots, src/kernels/prefill.rs:
// 48-87).  The exact int32 block dots of (token m, row n, block b) come from
// the tensor cores, 128 tokens x 128 rows per CTA tile:
//   TQ2_0: weights c - 1 in -1..2 (s8; code 3 decodes to +2) x Q8_K codes (s8)
//   Q2_K : isum = sum(sc*q * a) with sc*q in 0..45 (u8), K = 256;
//          msum = sum_g sums_g * min_g as one more K = 32 product: with
//          sums_g = 16*hi_g + lo_g (lo in 0..15, hi in -127..127, both s8),
//          msum = sum_g lo_g*min_g + hi_g*(16*min_g), 16*min_g <= 240 (u8).
//
// Pipeline per CTA (warp-specialised, see gemm_tokens_kernel): a load
// thread stages each block with bulk copies into one of three load stages --
// the tokens' Q8_K codes (128 x 256 B, stored tile-major by the quantize
// kernel in the K-major core-matrix layout: 8 rows x 16 B per core matrix,
// K-adjacent core matrices 2 KB apart, row-adjacent ones 128 B) and the
// packed weight units of the 128 rows; four warps expand the 2-bit codes
// into 8-bit core matrices (two unpack stages); one thread issues the MMAs
// into one of two TMEM accumulators; eight warps read finished accumulators
// (tcgen05.ld) and extend the binary32 chains on the CUDA cores.  All hand-
// offs are mbarriers, so loads, unpacking, MMAs and epilogues of successive
// blocks overlap.
#pragma once

#include "common.cuh"
#include "executor.cuh"
#include "matvec.cuh"
#include "q8k.cuh"

namespace prism {

constexpr int kGemmM = 128;       // tokens per CTA tile
constexpr int kGemmN = 128;       // weight rows per CTA tile
constexpr int kGemmThreads = 448;  // 14 warps, roles below
constexpr int kGemmLoadStages = 3;
constexpr int kMaxTokens = 1 << 16;  // tokens per multi-token projection call

// ---- token activations prepared once: Q8_K per (token, block) --------------
// Codes and split sums are stored tile-major, already in the tensor cores'
// K-major core-matrix order: for token tile t = m / 128 and block b, one
// contiguous 32 KB run [16-byte chunk kc][row m % 128][16 B] of codes and
// one 4 KB run [2][128][16 B] of split sums, so that a single bulk copy
// stages an operand.
struct TokenQ8K {
  int8_t *codes;     // [M/128 padded][nb][16][128][16]
  float *scale;      // [M][nb]
  int8_t *split;     // [M/128 padded][nb][2][128][16]  lo_g | hi_g of the group sums
};

__host__ __device__ inline size_t token_tile(int m, int nb, int b) {
  return (size_t)(m / 128) * nb + b;
}

// Store one quantized (token, block) unit: the lane holds codes
// 8*lane..8*lane+7 (w0, w1), the pair sum of its 16-group half and, on lane
// 0, the block scale.
__device__ __forceinline__ void store_token_unit(const TokenQ8K &out, int nb, int m, int b,
                                                 int lane, uint32_t w0, uint32_t w1, int pair,
                                                 float scale) {
  // lane holds codes 8*lane..8*lane+7: chunk kc = lane/2, half lane%2
  const size_t tile = token_tile(m, nb, b);
  const int row = m & 127;
  *reinterpret_cast<uint2 *>(out.codes + tile * 32768 + (lane >> 1) * 2048 + row * 16 +
                             (lane & 1) * 8) = make_uint2(w0, w1);
  if ((lane & 1) == 0) {
    // |pair| <= 16 * 127: lo = pair mod 16 in 0..15, hi = floor(pair / 16) in -127..127
    int8_t *sp = out.split + tile * 4096 + row * 16;
    sp[lane >> 1] = (int8_t)(pair & 15);
    sp[2048 + (lane >> 1)] = (int8_t)(pair >> 4);
  }
  if (lane == 0) out.scale[(size_t)m * nb + b] = scale;
}

// Quantize one (token, block) of x (row stride nb * 256 floats); returns
// the packed codes in w0/w1 plus the pair sum and scale.
__device__ __forceinline__ void quantize_token_unit(const float *__restrict__ x, int nb, int m,
                                                    int b, int lane, int pinned, uint32_t &w0,
                                                    uint32_t &w1, int &pair, float &scale,
                                                    unsigned *status) {
  const float *src = x + (size_t)m * nb * 256 + b * 256 + lane * 8;
  const float4 a = reinterpret_cast<const float4 *>(src)[0];
  const float4 c = reinterpret_cast<const float4 *>(src)[1];
  const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
  int8_t q[8];
  const unsigned st = q8k_quantize_regs(v, lane, pinned != 0, scale, q, pair);
  if (st && lane == 0) report(status, st);
  w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) |
       ((uint32_t)(uint8_t)q[2] << 16) | ((uint32_t)(uint8_t)q[3] << 24);
  w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) |
       ((uint32_t)(uint8_t)q[6] << 16) | ((uint32_t)(uint8_t)q[7] << 24);
}

// one warp per (token, block); reference q8k_with_input (src/kernels.rs:463-522)
__global__ void __launch_bounds__(256) q8k_tokens_kernel(const float *__restrict__ x, int M,
                                                         int nb, int pinned, TokenQ8K out,
                                                         unsigned *status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  grid_dependency_wait();
  grid_dependents_launch();
  if (warp >= M * nb) return;
  const int m = warp / nb, b = warp % nb;
  uint32_t w0, w1;
  int pair;
  float scale;
  quantize_token_unit(x, nb, m, b, lane, pinned, w0, w1, pair, scale, status);
  store_token_unit(out, nb, m, b, lane, w0, w1, pair, scale);
}

// ---- tcgen05 helpers (PTX ISA: tensor memory, matrix and instruction
// descriptors) ----------------------------------------------------------------

// Shared-memory matrix descriptor, K-major, no swizzle: start address,
// leading-dimension (K-adjacent core matrix) and stride-dimension
// (row-adjacent core matrix) byte offsets, all >> 4; version 1.
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;                // base offset 0, legacy LBO mode, SWIZZLE_NONE
}

// Instruction descriptor, kind::i8: D s32, A s8 (activations), B u8
// (weight codes), both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
  return (2u << 4)                       // D format: s32
         | (1u << 7)                     // A format: signed 8-bit
         | (0u << 10)                    // B format: unsigned 8-bit
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 32 lanes x 32 bits, 32 consecutive columns per thread
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// ---- tensor-parallel exchanges over peer memory ---------------------------
// A producer stores its output straight into every rank's buffer (peer
// memory mapped over NVLink, this rank's own included), then, after a
// system-scope fence, adds the number of values it delivered to each rank's
// arrival counter.  Counters only grow: a consumer waits until its counter
// reaches steps_completed * per_step + offset, where per_step is what one
// step delivers and offset what this step has delivered up to and including
// the awaited exchange.
constexpr int kMaxTp = 8;

struct TpWait {
  const unsigned long long *count;  // this rank's arrival counter (null: no wait)
  const unsigned long long *xstep;  // steps completed on this rank
  unsigned long long per_step, offset;
};

// Bounded wait (one thread); false when it expired, or when an earlier wait
// of this executor already did (the step has failed: do not wait again).
__device__ __forceinline__ bool tp_wait(const TpWait &w, unsigned *status) {
  if (*reinterpret_cast<volatile unsigned *>(status) & kStatusTimeout) return false;
  const unsigned long long target = *w.xstep * w.per_step + w.offset;
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

// Publish one CTA's deliveries: all of its stores are visible system-wide
// before any counter moves.  Called by every thread of the CTA.
__device__ __forceinline__ void tp_publish(unsigned long long *const *count, int ranks,
                                           unsigned long long delivered) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < ranks; ++p) atomicAdd_system(count[p], delivered);
  }
}

// The GEMM output sent to every rank: element (m, n) of the CTA's tile goes
// to dst[p][m * ld + col + n] of each rank p -- a row-parallel partial into
// rank p's receive slot for this rank, or (with the residual added) this
// rank's rows of the hidden state into rank p's copy.
struct GemmPush {
  float *dst[kMaxTp];
  unsigned long long *count[kMaxTp];  // rank p's arrival counter
  int n;                              // ranks (0: no exchange, store Y)
  int ld, col;
};

struct GemmArgs {
  const int8_t *codes;    // tile-major Q8_K codes (TokenQ8K)
  const int8_t *split;    // tile-major split group sums
  const uint8_t *w;       // tiled weight units (matvec.cuh layout)
  int h, nb, rows, ntiles;
  const float *scale;     // [M][nb]
  int M;
  float *y;               // [M][rows], or null
  const float *residual;  // optional [M][rows]: y = residual + chain (may alias y)
  unsigned long long *argmax_keys;  // optional [M]: greedy key over each token's rows
  int row_base;           // index of row 0 in the argmax key (a vocabulary slice's offset)
  unsigned *status;
  GemmPush push;
  TpWait gate;            // activations gathered from every rank: wait for them first
};

// Warp roles of the 14-warp CTA.
constexpr int kWarpUnpack = 1;  // warps 1..4: one weight row per thread
constexpr int kWarpMma = 5;     // lane 0 issues the MMAs
constexpr int kWarpEpi = 6;     // warps 6..13: epilogue (token lanes x 64 rows)

// Shared-memory layout of one CTA.
template <int KIND>
struct GemmSmem {
  static constexpr int kBlockBytes = KIND == 35 ? 66 : 84;
  // load stage: A codes 32 KB | A split 4 KB | packed weight units
  static constexpr int kA = 0, kA2 = 32768, kBp = 36864;
  static constexpr int kLoadStage = (kBp + kGemmN * kBlockBytes + 1023) / 1024 * 1024;
  // unpack stage: B codes 32 KB | B mins 4 KB
  static constexpr int kUnpack = kGemmLoadStages * kLoadStage;
  static constexpr int kBu = 0, kB2 = 32768;
  static constexpr int kUnpackStage = 36864;
  // ring of 4: d[128], dmin[128] of each block's rows (f32)
  static constexpr int kScales = kUnpack + 2 * kUnpackStage;
  static constexpr int kBars = kScales + 4096;
  static constexpr int kBytes = kBars + 256;
  static constexpr int kTmemCols = KIND == 35 ? 256 : 512;  // 2 x (isum [+ msum]) x 128
};

// Core-matrix offset (bytes) of (row, 16-byte K chunk) within a 128-row
// K-major tile.
__device__ __forceinline__ int core_off(int row, int kc) {
  return kc * 2048 + (row >> 3) * 128 + (row & 7) * 16;
}

// Warp-specialised CTA (448 threads):
//   warp 0 lane 0  issues each block's bulk copies once its load stage is
//                  free (lfree: the MMAs that read it completed);
//   warps 1..4     unpack a block's weight rows into u8/s8 core matrices once
//                  the copies landed (full) and the unpack stage is free
//                  (ufree), then arrive on ufull;
//   warp 5 lane 0  waits ufull and a drained accumulator (aempty), issues the
//                  MMAs, publishes the block's scales (dready) and commits
//                  afull / ufree / lfree;
//   warps 6..13    wait dready + afull, read TMEM and extend the chains, then
//                  arrive on aempty.
// Every wait is bounded; a role that gives up raises the CTA's fail flag and
// the others stop at their next wait.
template <int KIND>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tokens_kernel(const __grid_constant__ GemmArgs g) {
  using L = GemmSmem<KIND>;
  extern __shared__ __align__(1024) uint8_t gsm[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(gsm + L::kBars);
  uint64_t *full = bars, *lfree = bars + 3;                  // [3] each
  uint64_t *ufull = bars + 6, *ufree = bars + 8;             // [2] each
  uint64_t *afull = bars + 10, *aempty = bars + 12;          // [2] each
  uint64_t *dready = bars + 14;                              // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);
  volatile int *fail = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *dring = reinterpret_cast<float *>(gsm + L::kScales);  // [4][128]
  float *mring = dring + 4 * kGemmN;                           // [4][128]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kGemmN, m0 = blockIdx.y * kGemmM;
  const int nb = g.nb, h = g.h;
  const int unit = unit_bytes(KIND, h);
  const int tile0 = n0 / h, tiles = kGemmN / h;

  if (warp == 0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < 3; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&lfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ufull[i], 4 * 32);
      mbar_init(&ufree[i], 1);
      mbar_init(&afull[i], 1);
      mbar_init(&aempty[i], 8 * 32);
      mbar_init(&dready[i], 1);
    }
    *fail = 0;
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();
  grid_dependents_launch();
  if (g.gate.count) {
    // a gathered activation: every rank's blocks must have landed
    if (tid == 0 && !tp_wait(g.gate, g.status)) *fail = 1;
    __syncthreads();
  }

  float acc[64];
#pragma unroll
  for (int c = 0; c < 64; ++c) acc[c] = 0.0f;

  if (*fail) {
    // the gathered activations never arrived: no role runs
  } else if (warp == 0) {
    // ---- loads -------------------------------------------------------------
    if (lane == 0) {
      int copies = 0;
      for (int i = 0; i < tiles; ++i) copies += tile0 + i < g.ntiles;
      const uint32_t bytes = 32768u + (KIND == 10 ? 4096u : 0u) + (uint32_t)(copies * unit);
      for (int b = 0; b < nb; ++b) {
        const int ls = b % kGemmLoadStages;
        if (b >= kGemmLoadStages &&
            !mbar_wait_bounded(&lfree[ls], (unsigned)(b / kGemmLoadStages - 1) & 1u, g.status))
          *fail = 1;
        if (*fail) break;
        uint8_t *st = gsm + ls * L::kLoadStage;
        const size_t tile = token_tile(m0, nb, b);
        mbar_arrive_expect_tx(&full[ls], bytes);
        bulk_g2s(st + L::kA, g.codes + tile * 32768, 32768u, &full[ls]);
        if (KIND == 10) bulk_g2s(st + L::kA2, g.split + tile * 4096, 4096u, &full[ls]);
        for (int i = 0; i < tiles; ++i)
          if (tile0 + i < g.ntiles)
            bulk_g2s(st + L::kBp + i * unit, g.w + ((size_t)(tile0 + i) * nb + b) * unit, unit,
                     &full[ls]);
      }
    }
  } else if (warp < kWarpMma) {
    // ---- unpack: thread = weight row ---------------------------------------
    const int row = tid - 32 * kWarpUnpack, n = n0 + row;
    const bool valid = n < g.rows;
    const int r = row % h;
    for (int b = 0; b < nb; ++b) {
      const int ls = b % kGemmLoadStages, us = b & 1;
      bool ok = mbar_wait_bounded(&full[ls], (unsigned)(b / kGemmLoadStages) & 1u, g.status);
      if (ok && b >= 2) ok = mbar_wait_bounded(&ufree[us], (unsigned)(b / 2 - 1) & 1u, g.status);
      if (!ok) *fail = 1;
      if (*fail) break;
      const uint8_t *u = gsm + ls * L::kLoadStage + L::kBp + (row / h) * unit;
      uint8_t *ust = gsm + L::kUnpack + us * L::kUnpackStage;
      uint4 scv = make_uint4(0u, 0u, 0u, 0u);
      if (KIND == 10 && valid) scv = *reinterpret_cast<const uint4 *>(u + 64 * h + r * 16);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 wq = make_uint4(0u, 0u, 0u, 0u);
        if (valid) wq = *reinterpret_cast<const uint4 *>(u + (c * h + r) * 16);
        // packed chunk c holds, in bit plane j, the 16 codes of K chunk
        // kc = (c/2)*8 + 2j + (c%2)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const unsigned mk = 0x03030303u << (2 * j);
          uint4 o = make_uint4((wq.x & mk) >> (2 * j), (wq.y & mk) >> (2 * j),
                               (wq.z & mk) >> (2 * j), (wq.w & mk) >> (2 * j));
          const int kc = (c >> 1) * 8 + 2 * j + (c & 1);
          if (KIND == 35) {
            // signed ternary weights: code - 1 per byte (code 3 -> +2)
            o.x = __vsub4(o.x, 0x01010101u);
            o.y = __vsub4(o.y, 0x01010101u);
            o.z = __vsub4(o.z, 0x01010101u);
            o.w = __vsub4(o.w, 0x01010101u);
          } else {
            const unsigned sc = byte_of(scv, kc) & 15u;  // sc*q <= 45: no byte carries
            o.x *= sc;
            o.y *= sc;
            o.z *= sc;
            o.w *= sc;
          }
          *reinterpret_cast<uint4 *>(ust + L::kBu + core_off(row, kc)) = o;
        }
      }
      float d = 0.0f, dm = 0.0f;
      if (valid) {
        if (KIND == 35) {
          d = half_bits_to_float(reinterpret_cast<const uint16_t *>(u + 64 * h)[r]);
        } else {
          const uint16_t *dd = reinterpret_cast<const uint16_t *>(u + 80 * h);
          d = half_bits_to_float(dd[r]);
          dm = half_bits_to_float(dd[h + r]);
        }
      }
      dring[(b & 3) * kGemmN + row] = d;
      mring[(b & 3) * kGemmN + row] = dm;
      if (KIND == 10) {
        // B mins, K = 32: chunk 0 = min_g, chunk 1 = 16*min_g (g = 0..15)
        const uint4 lo = make_uint4((scv.x >> 4) & 0x0f0f0f0fu, (scv.y >> 4) & 0x0f0f0f0fu,
                                    (scv.z >> 4) & 0x0f0f0f0fu, (scv.w >> 4) & 0x0f0f0f0fu);
        const uint4 hi = make_uint4(lo.x << 4, lo.y << 4, lo.z << 4, lo.w << 4);
        *reinterpret_cast<uint4 *>(ust + L::kB2 + core_off(row, 0)) = lo;
        *reinterpret_cast<uint4 *>(ust + L::kB2 + core_off(row, 1)) = hi;
      }
      fence_proxy_async_smem();  // generic stores -> tensor-core (async proxy) reads
      mbar_arrive(&ufull[us]);
    }
  } else if (warp == kWarpMma) {
    // ---- MMA issue -----------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc =
          umma_idesc_i8(kGemmM, kGemmN) | (KIND == 35 ? (1u << 10) : 0u);  // TQ2_0: B s8
      constexpr uint32_t idesc_min = umma_idesc_i8(kGemmM, kGemmN);
      for (int b = 0; b < nb; ++b) {
        const int ls = b % kGemmLoadStages, us = b & 1;
        bool ok = mbar_wait_bounded(&ufull[us], (unsigned)(b / 2) & 1u, g.status);
        if (ok && b >= 2) ok = mbar_wait_bounded(&aempty[us], (unsigned)(b / 2 - 1) & 1u, g.status);
        if (!ok) *fail = 1;
        if (*fail) break;
        mbar_arrive(&dready[us]);  // the block's scales are in place
        tc_fence_after();
        const uint32_t a = smem_addr(gsm + ls * L::kLoadStage + L::kA);
        const uint32_t bsm = smem_addr(gsm + L::kUnpack + us * L::kUnpackStage + L::kBu);
        const uint32_t accd = tmem + (uint32_t)(us * (L::kTmemCols / 2));
#pragma unroll
        for (int k = 0; k < 8; ++k)  // K step k: chunks 2k, 2k+1
          umma_i8(accd, umma_smem_desc(a + k * 4096, 2048, 128),
                  umma_smem_desc(bsm + k * 4096, 2048, 128), idesc, k > 0 ? 1u : 0u);
        if (KIND == 10)
          umma_i8(accd + kGemmN, umma_smem_desc(a + L::kA2, 2048, 128),
                  umma_smem_desc(bsm + L::kB2, 2048, 128), idesc_min, 0u);
        umma_commit(&afull[us]);
        umma_commit(&ufree[us]);
        umma_commit(&lfree[ls]);
      }
    }
  } else {
    // ---- epilogue: thread = token, 64 rows ----------------------------------
    const int q4 = warp & 3, half = (warp - kWarpEpi) >> 2;
    const int m = m0 + 32 * q4 + lane;
    const bool mvalid = m < g.M;
    float sa_next = mvalid ? g.scale[(size_t)m * nb] : 0.0f;
    for (int b = 0; b < nb; ++b) {
      const int us = b & 1;
      const float sa = sa_next;
      if (mvalid && b + 1 < nb) sa_next = g.scale[(size_t)m * nb + b + 1];
      bool ok = mbar_wait_bounded(&dready[us], (unsigned)(b / 2) & 1u, g.status);
      if (ok) ok = mbar_wait_bounded(&afull[us], (unsigned)(b / 2) & 1u, g.status);
      if (!ok) *fail = 1;
      if (*fail) break;
      tc_fence_after();
      const float *dsc = dring + (b & 3) * kGemmN + 64 * half;
      const float *dmn = mring + (b & 3) * kGemmN + 64 * half;
      const uint32_t base =
          tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(us * (L::kTmemCols / 2) + 64 * half);
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        uint32_t rv[16];
        tmem_ld16(base + (uint32_t)(16 * part), rv);
        if (KIND == 35) {
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int cc = 16 * part + c;
            acc[cc] = __fadd_rn(acc[cc], __fmul_rn((float)(int)rv[c], __fmul_rn(dsc[cc], sa)));
          }
        } else {
          uint32_t mv[16];
          tmem_ld16(base + (uint32_t)(kGemmN + 16 * part), mv);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int cc = 16 * part + c;
            const float t1 = __fmul_rn(__fmul_rn(sa, dsc[cc]), (float)(int)rv[c]);
            const float t2 = __fmul_rn(__fmul_rn(sa, dmn[cc]), (float)(int)mv[c]);
            acc[cc] = __fadd_rn(acc[cc], __fsub_rn(t1, t2));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&aempty[us]);
    }
  }

  // ---- outputs: 128 x 128 tile through shared memory (row pitch 129) ------
  constexpr int kPitch = kGemmN + 1;
  float *otile = reinterpret_cast<float *>(gsm);
  tc_fence_before();
  __syncthreads();
  const bool ok = *fail == 0;
  if (ok && warp >= kWarpEpi) {
    const int q4 = warp & 3, half = (warp - kWarpEpi) >> 2;
    const int tl = 32 * q4 + lane;
    bool finite = true;
    unsigned long long best = 0ull;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      const int n = n0 + 64 * half + c;
      otile[tl * kPitch + 64 * half + c] = acc[c];
      if (n < g.rows) {
        finite &= is_finite_f(acc[c]);
        const unsigned long long key = argmax_key(acc[c], g.row_base + n);
        best = key > best ? key : best;
      }
    }
    if (m0 + tl < g.M) {
      if (!finite && !g.residual) report(g.status, kStatusNonfinite);
      if (g.argmax_keys && best) atomicMax(&g.argmax_keys[m0 + tl], best);
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
  if (ok && g.push.n) {
    // coalesced 512-byte rows into every rank's buffer
    for (int i = tid; i < kGemmM * kGemmN; i += kGemmThreads) {
      const int t = i / kGemmN, c = i % kGemmN;
      const int mm = m0 + t, n = n0 + c;
      if (mm < g.M && n < g.rows) {
        const size_t at = (size_t)mm * g.push.ld + g.push.col + n;
        float v = otile[t * kPitch + c];
        if (g.residual) {
          v = __fadd_rn(g.residual[at], v);
          if (!is_finite_f(v)) report(g.status, kStatusNonfinite);
        }
        for (int p = 0; p < g.push.n; ++p) g.push.dst[p][at] = v;
      }
    }
  } else if (ok) {
    for (int i = tid; i < kGemmM * kGemmN; i += kGemmThreads) {
      const int t = i / kGemmN, c = i % kGemmN;
      const int mm = m0 + t, n = n0 + c;
      if (mm < g.M && n < g.rows) {
        float v = otile[t * kPitch + c];
        if (g.residual) {
          v = __fadd_rn(g.residual[(size_t)mm * g.rows + n], v);
          if (!is_finite_f(v)) report(g.status, kStatusNonfinite);
        }
        if (g.y) g.y[(size_t)mm * g.rows + n] = v;
      }
    }
  }
  if (g.push.n) {
    // a failed CTA still counts, so that no rank waits out its limit; its
    // own status word carries the failure
    const unsigned long long tm = (unsigned long long)min(kGemmM, g.M - m0);
    const unsigned long long tn = (unsigned long long)min(kGemmN, g.rows - n0);
    tp_publish(g.push.count, g.push.n, tm * tn);
  }
}

// ---- host side -----------------------------------------------------------

template <int KIND>
constexpr int gemm_smem_bytes() {
  return GemmSmem<KIND>::kBytes;
}

// Quantize M token rows of x [M][nb*256] to Q8_K (tile-major, TokenQ8K).
inline cudaError_t launch_token_quantize(const float *x, size_t M, int nb, int pinned,
                                         const TokenQ8K &t, unsigned *status, cudaStream_t s,
                                         bool pdl) {
  cudaLaunchAttribute attr[1];
  const long warps = (long)M * nb;
  cudaLaunchConfig_t cfg =
      pdl_config(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, q8k_tokens_kernel, x, (int)M, nb, pinned, t, status);
}

// Y[M][rows] (= residual + chain when residual is set) for quantized tokens
// t; with argmax_keys, each token's greedy key over the rows.
inline cudaError_t launch_token_matmul(const DeviceWeight &dw, size_t M, const TokenQ8K &t,
                                       float *y, const float *residual,
                                       unsigned long long *argmax_keys, unsigned *status,
                                       cudaStream_t s, bool pdl, const GemmPush *push = nullptr,
                                       int row_base = 0, const TpWait *gate = nullptr) {
  GemmArgs g;
  g.codes = t.codes;
  g.split = t.split;
  g.w = dw.units;
  g.h = dw.h;
  g.nb = dw.nb;
  g.rows = (int)dw.rows;
  g.ntiles = dw.ntiles;
  g.scale = t.scale;
  g.M = (int)M;
  g.y = y;
  g.residual = residual;
  g.argmax_keys = argmax_keys;
  g.row_base = 0;
  g.status = status;
  g.push.n = 0;
  g.gate.count = nullptr;
  if (push) g.push = *push;
  if (gate) g.gate = *gate;
  if (row_base) g.row_base = row_base;
  void (*kernel)(GemmArgs) = dw.kind == 35 ? gemm_tokens_kernel<35> : gemm_tokens_kernel<10>;
  const int smem = dw.kind == 35 ? gemm_smem_bytes<35>() : gemm_smem_bytes<10>();
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)((dw.rows + kGemmN - 1) / kGemmN),
                                           (unsigned)((M + kGemmM - 1) / kGemmM)),
                                      dim3(kGemmThreads), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, kernel, g);
}

// Quantize M token rows of x [M][cols] to Q8_K, then Y[M][rows] = tokens x W^T
// on the tensor cores.  Both kernels go on `s` in order.
inline cudaError_t launch_token_gemm(const DeviceWeight &dw, const float *x, size_t M,
                                     int pinned, const TokenQ8K &t, float *y, unsigned *status,
                                     cudaStream_t s, bool pdl) {
  cudaError_t e = launch_token_quantize(x, M, dw.nb, pinned, t, status, s, pdl);
  if (e != cudaSuccess) return e;
  return launch_token_matmul(dw, M, t, y, nullptr, nullptr, status, s, pdl);
}

// Bytes of the token activation buffers for M tokens of nb blocks, and the
// carve of one buffer into them (codes and split stay 16-byte aligned).
inline size_t token_q8k_bytes(size_t M, int nb) {
  const size_t mpad = (M + kGemmM - 1) / kGemmM * kGemmM;
  return mpad * nb * 256 + mpad * nb * 32 + M * nb * 4;
}
inline TokenQ8K token_q8k_carve(void *buf, size_t M, int nb) {
  const size_t mpad = (M + kGemmM - 1) / kGemmM * kGemmM;
  uint8_t *base = static_cast<uint8_t *>(buf);
  TokenQ8K t;
  t.codes = reinterpret_cast<int8_t *>(base);
  t.split = reinterpret_cast<int8_t *>(base + mpad * nb * 256);
  t.scale = reinterpret_cast<float *>(base + mpad * nb * 256 + mpad * nb * 32);
  return t;
}

}  // namespace prism
