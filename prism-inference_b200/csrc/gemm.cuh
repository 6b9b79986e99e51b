// gemm.cuh -- multi-token packed projection (prefill, batched decode) on the
// 5th-generation tensor cores: tcgen05.mma kind::i8 with TMEM accumulators.
//
// Y[m][n] = sum_b term(m, n, b) over the 256-column blocks b, the reference's
// sequential binary32 chain per output (TQ2_0: src/kernels/tquants.rs:270-287;
// Q2_K: src/kernels/kquants.rs:346-420), here for every token m of a tile
// (the reference's ProjectionTile per-token dots, src/kernels/prefill.rs:
// 48-87).  The exact int32 block dot of (token m, row n, block b) is one
// 128 x 128 x 256 tensor-core product per block:
//   TQ2_0: codes c in {0,1,2} (u8) x Q8_K codes (s8); int = C - sum(a)
//   Q2_K : sc*q in 0..45 (u8) x Q8_K codes (s8) = the scaled integer sum;
//          the min term sum_g sums_g*min_g is added on the CUDA cores.
//
// CTA tile 128 tokens x 128 rows.  Per block: the Q8_K codes of 128 tokens
// (32 KB) and the 2-bit codes of 128 weight rows, unpacked to u8 (32 KB),
// are written to shared memory as K-major "core matrices" (8 rows x 16
// bytes, no swizzle: the K-adjacent core matrix is 2048 B away, the
// row-adjacent one 128 B); one elected thread issues 8 MMAs (K = 32 each)
// into one of two TMEM int32 accumulators and commits to an mbarrier; the
// 8 warps read the finished accumulator with tcgen05.ld (warp w: lanes
// 32(w%4).., columns 64(w/4)..) and extend their binary32 chains while the
// next block's MMAs run.  Stages, accumulators and chains are double
// buffered.
#pragma once

#include "common.cuh"
#include "executor.cuh"
#include "matvec.cuh"
#include "q8k.cuh"

namespace prism {

constexpr int kGemmM = 128;       // tokens per CTA tile
constexpr int kGemmN = 128;       // weight rows per CTA tile
constexpr int kGemmThreads = 256;
constexpr int kGemmStage = kGemmM * 256 + kGemmN * 256;   // A + B bytes per block
constexpr int kGemmTmemCols = 256;                        // 2 x 128 int32 columns

// ---- token activations prepared once: Q8_K per (token, block) --------------
struct TokenQ8K {
  int8_t *codes;     // [M][K]
  float *scale;      // [M][nb]
  int *asum;         // [M][nb]   sum of the block's codes
  int16_t *sums;     // [M][nb][16]
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
  if ((lane & 1) == 0) out.sums[((size_t)m * nb + b) * 16 + (lane >> 1)] = (int16_t)pair;
  int tot = pair;
#pragma unroll
  for (int off = 2; off < 32; off <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (lane == 0) {
    out.scale[(size_t)m * nb + b] = scale;
    out.asum[(size_t)m * nb + b] = tot;
  }
}

// ---- tcgen05 helpers (PTX ISA: tensor memory, matrix/instruction descriptors)

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
// (weight codes), both K-major, M = 128, N = 128.
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

struct GemmArgs {
  const uint8_t *w;      // tiled weight units (matvec.cuh layout)
  int h, nb, rows;       // weight tile height, blocks per row, rows (N)
  TokenQ8K act;          // token activations
  int M;                 // tokens
  float *y;              // [M][rows]
  unsigned *status;
};

// Core-matrix offset (bytes) of (row, 16-byte K chunk) within a 128 x 256 B
// K-major tile.
__device__ __forceinline__ int core_off(int row, int kc) {
  return (kc * 16 + (row >> 3)) * 128 + (row & 7) * 16;
}

template <int KIND>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tokens_kernel(GemmArgs g) {
  extern __shared__ __align__(128) uint8_t gsm[];
  uint8_t *stage[2] = {gsm, gsm + kGemmStage};
  // per stage: A at +0 (128 x 256 B), B at +32768 (128 x 256 B)
  float *dsc = reinterpret_cast<float *>(gsm + 2 * kGemmStage);         // [2][128] d
  float *dmn = dsc + 2 * kGemmN;                                         // [2][128] dmin
  uint8_t *mins = reinterpret_cast<uint8_t *>(dmn + 2 * kGemmN);       // [2][128][16]
  uint64_t *bars = reinterpret_cast<uint64_t *>(mins + 2 * kGemmN * 16); // [2]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kGemmN, m0 = blockIdx.y * kGemmM;
  const int nb = g.nb;
  const int unit = unit_bytes(KIND, g.h);

  if (warp == 0) {
    tmem_alloc(tmem_slot, kGemmTmemCols);
    tmem_relinquish();
  }
  if (tid < 2) {
    mbar_init(&bars[tid], 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();
  grid_dependents_launch();

  // stage block b into buffer s: Q8_K codes of 128 tokens, unpacked codes of
  // 128 weight rows, the rows' block scales (and Q2_K mins)
  auto load_block = [&](int b, int s) {
    uint8_t *A = stage[s], *B = stage[s] + kGemmM * 256;
    for (int i = tid; i < kGemmM * 16; i += kGemmThreads) {
      const int row = i >> 4, kc = i & 15, m = m0 + row;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (m < g.M)
        v = *reinterpret_cast<const uint4 *>(g.act.codes + (size_t)m * nb * 256 + b * 256 + kc * 16);
      *reinterpret_cast<uint4 *>(A + core_off(row, kc)) = v;
    }
    // packed chunk c (16 bytes) of a weight row holds, in plane j, the 16
    // codes of K chunk kc = (c/2)*8 + 2j + (c%2)
    for (int i = tid; i < kGemmN * 4; i += kGemmThreads) {
      const int row = i >> 2, c = i & 3, n = n0 + row;
      uint4 wq = make_uint4(0u, 0u, 0u, 0u);
      uint4 scv = make_uint4(0u, 0u, 0u, 0u);
      if (n < g.rows) {
        const uint8_t *u = g.w + ((size_t)(n / g.h) * nb + b) * unit;
        wq = *reinterpret_cast<const uint4 *>(u + (c * g.h + n % g.h) * 16);
        if (KIND == 10) scv = *reinterpret_cast<const uint4 *>(u + 64 * g.h + (n % g.h) * 16);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const unsigned mk = 0x03030303u << (2 * j);
        uint4 o = make_uint4((wq.x & mk) >> (2 * j), (wq.y & mk) >> (2 * j),
                             (wq.z & mk) >> (2 * j), (wq.w & mk) >> (2 * j));
        const int kc = (c >> 1) * 8 + 2 * j + (c & 1);
        if (KIND == 10) {
          // scale the 16 codes of group kc by its 4-bit scale (sc*q <= 45)
          const unsigned sc = byte_of(scv, kc) & 15u;
          o.x *= sc;
          o.y *= sc;
          o.z *= sc;
          o.w *= sc;
        }
        *reinterpret_cast<uint4 *>(B + core_off(row, kc)) = o;
      }
      if (c == 0) {
        float d = 0.0f, dm = 0.0f;
        if (n < g.rows) {
          const uint8_t *u = g.w + ((size_t)(n / g.h) * nb + b) * unit;
          if (KIND == 35) {
            d = half_bits_to_float(reinterpret_cast<const uint16_t *>(u + 64 * g.h)[n % g.h]);
          } else {
            const uint16_t *dd = reinterpret_cast<const uint16_t *>(u + 80 * g.h);
            d = half_bits_to_float(dd[n % g.h]);
            dm = half_bits_to_float(dd[g.h + n % g.h]);
          }
        }
        dsc[s * kGemmN + row] = d;
        dmn[s * kGemmN + row] = dm;
        if (KIND == 10) {
#pragma unroll
          for (int q = 0; q < 16; ++q) mins[(s * kGemmN + row) * 16 + q] = byte_of(scv, q) >> 4;
        }
      }
    }
    fence_proxy_async_smem();  // generic writes -> tensor-core (async proxy) reads
  };

  auto issue_mma = [&](int s) {
    const uint32_t a = smem_addr(stage[s]), bsm = smem_addr(stage[s] + kGemmM * 256);
    const uint32_t d = tmem + (uint32_t)(s * kGemmN);
    constexpr uint32_t idesc = umma_idesc_i8(kGemmM, kGemmN);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      // K step k covers 16-byte chunks 2k, 2k+1: 2 x 2048 B further along K
      const uint64_t ad = umma_smem_desc(a + k * 4096, 2048, 128);
      const uint64_t bd = umma_smem_desc(bsm + k * 4096, 2048, 128);
      umma_i8(d, ad, bd, idesc, k > 0 ? 1u : 0u);
    }
    umma_commit(&bars[s]);
  };

  // epilogue state: warp w covers tokens 32(w%4).. and rows 64(w/4)..
  const int q4 = warp & 3, half = warp >> 2;
  const int m = m0 + 32 * q4 + lane;
  float acc[64];
#pragma unroll
  for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
  bool failed = false;

  load_block(0, 0);
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
    issue_mma(0);
  }
  for (int b = 0; b < nb; ++b) {
    const int s = b & 1;
    if (b + 1 < nb) {
      // buffer s^1 was last read by block b-1's MMAs, completed before
      // that block's epilogue below released it
      load_block(b + 1, s ^ 1);
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_mma(s ^ 1);
      }
    }
    // epilogue of block b
    // every thread waits (bounded); all leave together if any gave up
    const bool done = mbar_wait_bounded(&bars[s], (unsigned)(b >> 1) & 1u, g.status);
    if (!__syncthreads_and(done)) {
      failed = true;
      break;
    }
    tc_fence_after();
    float sa = 0.0f;
    int asum = 0;
    int gsum[16];
    if (m < g.M) {
      sa = g.act.scale[(size_t)m * nb + b];
      asum = g.act.asum[(size_t)m * nb + b];
      if (KIND == 10) {
#pragma unroll
        for (int q = 0; q < 16; ++q) gsum[q] = g.act.sums[((size_t)m * nb + b) * 16 + q];
      }
    }
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q4) << 16) + (uint32_t)(s * kGemmN + 64 * half + 32 * part), r);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int col = 64 * half + 32 * part + c;
        const float d = dsc[s * kGemmN + col];
        const int v = (int)r[c];
        float term;
        if (KIND == 35) {
          term = __fmul_rn((float)(v - asum), __fmul_rn(d, sa));
        } else {
          const uint8_t *mn = mins + (s * kGemmN + col) * 16;
          int ms = 0;
#pragma unroll
          for (int q = 0; q < 16; ++q) ms += gsum[q] * (int)mn[q];
          const float t1 = __fmul_rn(__fmul_rn(sa, d), (float)v);
          const float t2 = __fmul_rn(__fmul_rn(sa, dmn[s * kGemmN + col]), (float)ms);
          term = __fsub_rn(t1, t2);
        }
        acc[32 * part + c] = __fadd_rn(acc[32 * part + c], term);
      }
    }
    tc_fence_before();
    __syncthreads();  // accumulator s and stage s are free again
  }
  // outputs: the 128 x 128 tile goes through shared memory (row pitch 129
  // floats) so that the global stores run along rows
  constexpr int kPitch = kGemmN + 1;
  float *otile = reinterpret_cast<float *>(gsm);
  if (!failed) {
    bool finite = true;
    const int tl = 32 * q4 + lane;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      otile[tl * kPitch + 64 * half + c] = acc[c];
      if (n0 + 64 * half + c < g.rows) finite &= is_finite_f(acc[c]);
    }
    if (m < g.M && !finite) report(g.status, kStatusNonfinite);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kGemmTmemCols);
  if (!failed) {
    for (int i = tid; i < kGemmM * kGemmN; i += kGemmThreads) {
      const int tl = i / kGemmN, c = i % kGemmN;
      const int mm = m0 + tl, n = n0 + c;
      if (mm < g.M && n < g.rows) g.y[(size_t)mm * g.rows + n] = otile[tl * kPitch + c];
    }
  }
}

__host__ __device__ constexpr int gemm_smem_bytes() {
  return 2 * kGemmStage + 2 * kGemmN * 4 * 2 + 2 * kGemmN * 16 + 2 * 8 + 16;
}

constexpr int kMaxTokens = 1 << 16;  // tokens per multi-token projection call

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
  g.w = dw.units;
  g.h = dw.h;
  g.nb = nb;
  g.rows = (int)dw.rows;
  g.act = t;
  g.M = (int)M;
  g.y = y;
  g.status = status;
  void (*kernel)(GemmArgs) =
      dw.kind == 35 ? gemm_tokens_kernel<35> : gemm_tokens_kernel<10>;
  const int smem = gemm_smem_bytes();
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cfg = pdl_config(dim3((unsigned)((dw.rows + kGemmN - 1) / kGemmN),
                        (unsigned)((M + kGemmM - 1) / kGemmM)),
                   dim3(kGemmThreads), smem, s, attr, pdl);
  return cudaLaunchKernelEx(&cfg, kernel, g);
}

}  // namespace prism
