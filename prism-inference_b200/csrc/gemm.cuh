// gemm.cuh -- multi-token packed projection (prefill, batched decode) on the
// 5th-generation tensor cores: tcgen05.mma kind::i8 with TMEM accumulators.
//
// Y[m][n] = sum_b term(m, n, b) over the 256-column blocks b, the reference's
// sequential binary32 chain per output (TQ2_0: src/kernels/tquants.rs:270-287;
// Q2_K: src/kernels/kquants.rs:346-420), here for every token m of a tile
// (the reference's ProjectionTile per-token dots, src/kernels/prefill.rs:
// 48-87).  The exact int32 block dots of (token m, row n, block b) come from
// the tensor cores, 128 tokens x 128 rows per CTA tile:
//   TQ2_0: raw codes c in 0..3 (u8) x Q8_K codes (s8); int = sum(c*a) - sum(a)
//   Q2_K : isum = sum(sc*q * a) with sc*q in 0..45 (u8), K = 256;
//          msum = sum_g sums_g * min_g as one more K = 32 product: with
//          sums_g = 16*hi_g + lo_g (lo in 0..15, hi in -127..127, both s8),
//          msum = sum_g lo_g*min_g + hi_g*(16*min_g), 16*min_g <= 240 (u8).
//
// Pipeline per CTA.  Three load stages, filled by one thread with TMA (the
// tokens' Q8_K codes, 128 x 256 B, straight into the K-major core-matrix
// layout: 8 rows x 16 B per core matrix, K-adjacent core matrices 2 KB
// apart, row-adjacent ones 128 B) and bulk copies (the packed weight units
// of the 128 rows).  Two unpack stages: all threads expand the 2-bit codes
// (and for Q2_K the scales and mins) into u8 core matrices, then one thread
// issues the MMAs into one of two TMEM accumulators and commits to an
// mbarrier.  The epilogue of block b-1 (tcgen05.ld, then the binary32
// chain on the CUDA cores; warp w owns TMEM lanes 32(w%4).. = tokens and
// columns 64(w/4).. = rows) runs while block b's MMAs execute, and block
// b+2's loads are in flight meanwhile.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "executor.cuh"
#include "matvec.cuh"
#include "q8k.cuh"

namespace prism {

constexpr int kGemmM = 128;       // tokens per CTA tile
constexpr int kGemmN = 128;       // weight rows per CTA tile
constexpr int kGemmThreads = 256;
constexpr int kGemmLoadStages = 3;
constexpr int kMaxTokens = 1 << 16;  // tokens per multi-token projection call

// ---- token activations prepared once: Q8_K per (token, block) --------------
struct TokenQ8K {
  int8_t *codes;     // [M][K]
  float *scale;      // [M][nb]
  int *asum;         // [M][nb]   sum of the block's codes
  int8_t *split;     // [M][nb][32]  lo_g (16 B) | hi_g (16 B) of the group sums
};

// one warp per (token, block); reference q8k_with_input (src/kernels.rs:463-522)
__global__ void __launch_bounds__(256) q8k_tokens_kernel(const float *__restrict__ x, int M,
                                                         int nb, int pinned, TokenQ8K out,
                                                         unsigned *status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  grid_dependency_wait();
  grid_dependents_launch();
  if (warp >= M * nb) return;
  const int m = warp / nb, b = warp % nb;
  const float *src = x + (size_t)m * nb * 256 + b * 256 + lane * 8;
  const float4 a = reinterpret_cast<const float4 *>(src)[0];
  const float4 c = reinterpret_cast<const float4 *>(src)[1];
  const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
  float scale;
  int8_t q[8];
  int pair;
  const unsigned st = q8k_quantize_regs(v, lane, pinned != 0, scale, q, pair);
  if (st && lane == 0) report(status, st);
  uint32_t w0 = (uint32_t)(uint8_t)q[0] | ((uint32_t)(uint8_t)q[1] << 8) |
                ((uint32_t)(uint8_t)q[2] << 16) | ((uint32_t)(uint8_t)q[3] << 24);
  uint32_t w1 = (uint32_t)(uint8_t)q[4] | ((uint32_t)(uint8_t)q[5] << 8) |
                ((uint32_t)(uint8_t)q[6] << 16) | ((uint32_t)(uint8_t)q[7] << 24);
  reinterpret_cast<uint2 *>(out.codes + (size_t)m * nb * 256 + b * 256)[lane] = make_uint2(w0, w1);
  if ((lane & 1) == 0) {
    // |pair| <= 16 * 128: lo = pair mod 16 in 0..15, hi = floor(pair / 16) in -128..127
    int8_t *sp = out.split + ((size_t)m * nb + b) * 32;
    sp[lane >> 1] = (int8_t)(pair & 15);
    sp[16 + (lane >> 1)] = (int8_t)(pair >> 4);
  }
  int tot = pair;
#pragma unroll
  for (int off = 2; off < 32; off <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (lane == 0) {
    out.scale[(size_t)m * nb + b] = scale;
    out.asum[(size_t)m * nb + b] = tot;
  }
}

// ---- tcgen05 / TMA helpers (PTX ISA: tensor memory, matrix and instruction
// descriptors, bulk tensor copies) ---------------------------------------------

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
// 3-D tiled TMA load into this CTA's shared memory (no multicast)
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

struct GemmArgs {
  CUtensorMap codes_map;  // Q8_K codes viewed as [K/16][M][16 B]
  CUtensorMap split_map;  // group-sum split viewed as [2 nb][M][16 B]
  const uint8_t *w;       // tiled weight units (matvec.cuh layout)
  int h, nb, rows, ntiles;
  const float *scale;     // [M][nb]
  const int *asum;        // [M][nb]
  int M;
  float *y;               // [M][rows]
  unsigned *status;
};

// Shared-memory layout of one CTA.
template <int KIND>
struct GemmSmem {
  static constexpr int kBlockBytes = KIND == 35 ? 66 : 84;
  // load stage: A codes 32 KB | A split 4 KB | packed weight units
  static constexpr int kA = 0, kA2 = 32768, kBp = 36864;
  static constexpr int kLoadStage = (kBp + kGemmN * kBlockBytes + 1023) / 1024 * 1024;
  // unpack stage: B codes 32 KB | B mins 4 KB | d[128] | dmin[128]
  static constexpr int kUnpack = kGemmLoadStages * kLoadStage;
  static constexpr int kBu = 0, kB2 = 32768, kD = 36864, kDmin = 37376;
  static constexpr int kUnpackStage = 37888;
  static constexpr int kBars = kUnpack + 2 * kUnpackStage;  // full[3], done[2], tmem slot
  static constexpr int kBytes = kBars + 64;
  static constexpr int kTmemCols = KIND == 35 ? 256 : 512;   // 2 x (isum [+ msum]) x 128
};

// Core-matrix offset (bytes) of (row, 16-byte K chunk) within a 128-row
// K-major tile.
__device__ __forceinline__ int core_off(int row, int kc) {
  return kc * 2048 + (row >> 3) * 128 + (row & 7) * 16;
}

template <int KIND>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tokens_kernel(const __grid_constant__ GemmArgs g) {
  using L = GemmSmem<KIND>;
  extern __shared__ __align__(1024) uint8_t gsm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(gsm + L::kBars);  // [3]
  uint64_t *done = full + kGemmLoadStages;                         // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kGemmN, m0 = blockIdx.y * kGemmM;
  const int nb = g.nb, h = g.h;
  const int unit = unit_bytes(KIND, h);
  const int tile0 = n0 / h, tiles = kGemmN / h;

  if (warp == 0) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < kGemmLoadStages + 2; ++i) mbar_init(&full[i], 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();
  grid_dependents_launch();

  // one thread: TMA the tokens' codes (and split sums), bulk-copy the rows'
  // packed units of block b into load stage b % 3
  auto issue_loads = [&](int b) {
    const int ls = b % kGemmLoadStages;
    uint8_t *st = gsm + ls * L::kLoadStage;
    int copies = 0;
    for (int i = 0; i < tiles; ++i) copies += tile0 + i < g.ntiles;
    const uint32_t bytes = 32768u + (KIND == 10 ? 4096u : 0u) + (uint32_t)(copies * unit);
    mbar_arrive_expect_tx(&full[ls], bytes);
    tma_load_3d(st + L::kA, &g.codes_map, 0, m0, b * 16, &full[ls]);
    if (KIND == 10) tma_load_3d(st + L::kA2, &g.split_map, 0, m0, b * 2, &full[ls]);
    for (int i = 0; i < tiles; ++i)
      if (tile0 + i < g.ntiles)
        bulk_g2s(st + L::kBp + i * unit, g.w + ((size_t)(tile0 + i) * nb + b) * unit, unit,
                 &full[ls]);
  };

  // all threads: expand block b's packed units (load stage b % 3) into u8
  // core matrices (unpack stage b % 2).  Thread t takes row t % 128 and the
  // packed chunks 2(t/128), 2(t/128)+1; eight consecutive threads write one
  // 128-byte run, so the stores are conflict-free.
  auto unpack = [&](int b) {
    const uint8_t *bp = gsm + (b % kGemmLoadStages) * L::kLoadStage + L::kBp;
    uint8_t *us = gsm + L::kUnpack + (b & 1) * L::kUnpackStage;
    const int row = tid & (kGemmN - 1), n = n0 + row;
    const bool valid = n < g.rows;
    const uint8_t *u = bp + (row / h) * unit;
    const int r = row % h;
    uint4 scv = make_uint4(0u, 0u, 0u, 0u);
    if (KIND == 10 && valid) scv = *reinterpret_cast<const uint4 *>(u + 64 * h + r * 16);
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * (tid >> 7) + cc;
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
        if (KIND == 10) {
          const unsigned sc = byte_of(scv, kc) & 15u;  // sc*q <= 45: no byte carries
          o.x *= sc;
          o.y *= sc;
          o.z *= sc;
          o.w *= sc;
        }
        *reinterpret_cast<uint4 *>(us + L::kBu + core_off(row, kc)) = o;
      }
    }
    if (tid < kGemmN) {
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
      reinterpret_cast<float *>(us + L::kD)[row] = d;
      reinterpret_cast<float *>(us + L::kDmin)[row] = dm;
    } else if (KIND == 10) {
      // B mins, K = 32: chunk 0 = min_g, chunk 1 = 16*min_g (g = 0..15)
      uint4 lo, hi;
      uint32_t *pl = reinterpret_cast<uint32_t *>(&lo), *ph = reinterpret_cast<uint32_t *>(&hi);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t wv = 0;
        if (valid) {
          const uint32_t s4 = q == 0 ? scv.x : q == 1 ? scv.y : q == 2 ? scv.z : scv.w;
          wv = (s4 >> 4) & 0x0f0f0f0fu;
        }
        pl[q] = wv;
        ph[q] = wv << 4;
      }
      *reinterpret_cast<uint4 *>(us + L::kB2 + core_off(row, 0)) = lo;
      *reinterpret_cast<uint4 *>(us + L::kB2 + core_off(row, 1)) = hi;
    }
  };

  auto issue_mma = [&](int b) {
    const uint8_t *st = gsm + (b % kGemmLoadStages) * L::kLoadStage;
    const uint8_t *us = gsm + L::kUnpack + (b & 1) * L::kUnpackStage;
    const uint32_t a = smem_addr(st + L::kA), bsm = smem_addr(us + L::kBu);
    const uint32_t acc = tmem + (uint32_t)((b & 1) * (L::kTmemCols / 2));
    constexpr uint32_t idesc = umma_idesc_i8(kGemmM, kGemmN);
#pragma unroll
    for (int k = 0; k < 8; ++k)  // K step k: chunks 2k, 2k+1
      umma_i8(acc, umma_smem_desc(a + k * 4096, 2048, 128),
              umma_smem_desc(bsm + k * 4096, 2048, 128), idesc, k > 0 ? 1u : 0u);
    if (KIND == 10)
      umma_i8(acc + kGemmN, umma_smem_desc(smem_addr(st + L::kA2), 2048, 128),
              umma_smem_desc(smem_addr(us + L::kB2), 2048, 128), idesc, 0u);
    umma_commit(&done[b & 1]);
  };

  // epilogue state: warp w covers tokens 32(w%4).. and rows 64(w/4)..
  const int q4 = warp & 3, half = warp >> 2;
  const int tl = 32 * q4 + lane, m = m0 + tl;
  const bool mvalid = m < g.M;
  float acc[64];
#pragma unroll
  for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
  bool failed = false;

  auto epilogue = [&](int b) -> bool {
    float sa = 0.0f;
    int asum = 0;
    if (mvalid) {
      sa = g.scale[(size_t)m * nb + b];
      asum = g.asum[(size_t)m * nb + b];
    }
    const bool ok = mbar_wait_bounded(&done[b & 1], (unsigned)(b >> 1) & 1u, g.status);
    if (!__syncthreads_and(ok)) return false;
    tc_fence_after();
    const uint8_t *us = gsm + L::kUnpack + (b & 1) * L::kUnpackStage;
    const float *dsc = reinterpret_cast<const float *>(us + L::kD);
    const float *dmn = reinterpret_cast<const float *>(us + L::kDmin);
    const uint32_t base =
        tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)((b & 1) * (L::kTmemCols / 2));
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const int col0 = 64 * half + 32 * part;
      uint32_t r[32];
      tmem_ld32(base + (uint32_t)col0, r);
      if (KIND == 35) {
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float term = __fmul_rn((float)((int)r[c] - asum), __fmul_rn(dsc[col0 + c], sa));
          acc[32 * part + c] = __fadd_rn(acc[32 * part + c], term);
        }
      } else {
        uint32_t ms[32];
        tmem_ld32(base + (uint32_t)(kGemmN + col0), ms);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float t1 = __fmul_rn(__fmul_rn(sa, dsc[col0 + c]), (float)(int)r[c]);
          const float t2 = __fmul_rn(__fmul_rn(sa, dmn[col0 + c]), (float)(int)ms[c]);
          acc[32 * part + c] = __fadd_rn(acc[32 * part + c], __fsub_rn(t1, t2));
        }
      }
    }
    return true;
  };

  if (tid == 0)
    for (int b = 0; b < kGemmLoadStages && b < nb; ++b) issue_loads(b);
  for (int b = 0; b < nb && !failed; ++b) {
    const bool ok = mbar_wait_bounded(&full[b % kGemmLoadStages],
                                      (unsigned)(b / kGemmLoadStages) & 1u, g.status);
    if (ok) unpack(b);
    fence_proxy_async_smem();  // generic stores -> tensor-core (async proxy) reads
    tc_fence_before();
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    if (tid == 0) {
      tc_fence_after();
      issue_mma(b);
    }
    if (b >= 1) {
      if (!epilogue(b - 1)) {
        failed = true;
        break;
      }
      tc_fence_before();
      __syncthreads();  // accumulator (b-1)&1 read; load stage (b-1)%3 consumed
      if (tid == 0 && b + 2 < nb) issue_loads(b + 2);
    }
  }
  if (!failed && !epilogue(nb - 1)) failed = true;

  // outputs: the 128 x 128 tile goes through shared memory (row pitch 129
  // floats) so that the global stores run along rows
  constexpr int kPitch = kGemmN + 1;
  float *otile = reinterpret_cast<float *>(gsm);
  tc_fence_before();
  __syncthreads();
  if (!failed) {
    bool finite = true;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      otile[tl * kPitch + 64 * half + c] = acc[c];
      if (n0 + 64 * half + c < g.rows) finite &= is_finite_f(acc[c]);
    }
    if (mvalid && !finite) report(g.status, kStatusNonfinite);
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::kTmemCols);
  if (!failed) {
    for (int i = tid; i < kGemmM * kGemmN; i += kGemmThreads) {
      const int t = i / kGemmN, c = i % kGemmN;
      const int mm = m0 + t, n = n0 + c;
      if (mm < g.M && n < g.rows) g.y[(size_t)mm * g.rows + n] = otile[t * kPitch + c];
    }
  }
}

// ---- host side -----------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// u8 tensor viewed as [d2][d1][16 B] with byte strides s1 (d1) and s2 (d2);
// box 16 x box1 x box2.
inline bool encode_rows16(CUtensorMap *map, const void *base, uint64_t d1, uint64_t d2,
                          uint64_t s1, uint64_t s2, uint32_t box1, uint32_t box2) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {16, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {16, box1, box2};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KIND>
constexpr int gemm_smem_bytes() {
  return GemmSmem<KIND>::kBytes;
}

// Quantize M token rows of x [M][cols] to Q8_K, then Y[M][rows] = tokens x W^T
// on the tensor cores.  Both kernels go on `s` in order.
inline cudaError_t launch_token_gemm(const DeviceWeight &dw, const float *x, size_t M,
                                     int pinned, const TokenQ8K &t, float *y, unsigned *status,
                                     cudaStream_t s, bool pdl) {
  const int nb = dw.nb;
  cudaLaunchAttribute attr[1];
  const long warps = (long)M * nb;
  cudaLaunchConfig_t cfg =
      pdl_config(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, s, attr, pdl);
  cudaError_t e = cudaLaunchKernelEx(&cfg, q8k_tokens_kernel, x, (int)M, nb, pinned, t, status);
  if (e != cudaSuccess) return e;
  GemmArgs g;
  memset(&g, 0, sizeof(g));
  if (!encode_rows16(&g.codes_map, t.codes, M, (uint64_t)nb * 16, (uint64_t)nb * 256, 16,
                     kGemmM, 16) ||
      !encode_rows16(&g.split_map, t.split, M, (uint64_t)nb * 2, (uint64_t)nb * 32, 16, kGemmM,
                     2))
    return cudaErrorInvalidValue;
  g.w = dw.units;
  g.h = dw.h;
  g.nb = nb;
  g.rows = (int)dw.rows;
  g.ntiles = dw.ntiles;
  g.scale = t.scale;
  g.asum = t.asum;
  g.M = (int)M;
  g.y = y;
  g.status = status;
  void (*kernel)(GemmArgs) = dw.kind == 35 ? gemm_tokens_kernel<35> : gemm_tokens_kernel<10>;
  const int smem = dw.kind == 35 ? gemm_smem_bytes<35>() : gemm_smem_bytes<10>();
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cfg = pdl_config(dim3((unsigned)((dw.rows + kGemmN - 1) / kGemmN),
                        (unsigned)((M + kGemmM - 1) / kGemmM)),
                   dim3(kGemmThreads), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, kernel, g);
}

}  // namespace prism
