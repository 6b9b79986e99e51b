// executor.cuh -- host-side executor state and kernel launch helpers shared
// by the C ABI translation units.  Not part of the public ABI.
#pragma once

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <set>
#include <string>

#include <cuda_runtime.h>

#include "../../include/prism_b200.h"
#include "matvec.cuh"
#include "q8k.cuh"

namespace prism {

// A projection weight resident in HBM in the tiled layout (matvec.cuh).
struct DeviceWeight {
  uint32_t kind = 0;
  uint64_t rows = 0, cols = 0;
  int nb = 0, h = 32, ntiles = 0;
  uint8_t *units = nullptr;
  uint64_t bytes = 0;   // device bytes of the tiled layout
  bool packed = false;  // PQ2 / PTQ1 rows as uploaded (packed.cuh), not tiled
};

// The double-buffered tile must also fit the 227 KB shared-memory budget.
constexpr int kMaxSmem = 232448;
constexpr int kSmPerSm = 233472;  // shared memory per SM

// Tile height: the largest of 32/16/8 rows that still gives every SM a tile
// (tiles of 32 rows use one lane per row; 16 and 8 split a row's four
// 16-byte chunks over 2 or 4 lanes).
inline int choose_tile_height(uint32_t kind, uint64_t rows, uint64_t cols, int num_sms) {
  int h = 8;
  if ((rows + 31) / 32 >= (uint64_t)2 * num_sms) h = 32;
  else if ((rows + 15) / 16 >= (uint64_t)num_sms) h = 16;
  const int nb = (int)(cols / 256);
  // sized for the up+gate pair (two tiles per buffer), the largest case
  while (h > 8 && MatvecSmem(nb, h, unit_bytes((int)kind, h), 2 * nb).total() > kMaxSmem) h /= 2;
  return h;
}

inline int packed_block_bytes(uint32_t kind) {
  return kind == 35 ? 66 : kind == 10 ? 84 : 0;
}

// Every fp16 block scale finite (reference `scale`, src/kernels.rs:152-154).
inline bool scales_finite(uint32_t kind, const uint8_t *src, size_t nblocks) {
  const int bb = packed_block_bytes(kind);
  for (size_t i = 0; i < nblocks; ++i) {
    const uint8_t *blk = src + i * bb;
    if (kind == 35) {
      if ((blk[65] & 0x7c) == 0x7c) return false;
    } else if ((blk[81] & 0x7c) == 0x7c || (blk[83] & 0x7c) == 0x7c) {
      return false;
    }
  }
  return true;
}

// Copy reference-layout packed rows to HBM and repack them into the tiled
// layout (matvec.cuh).  Synchronous on `s`.
inline cudaError_t upload_tiled(const uint8_t *host, uint32_t kind, uint64_t rows, uint64_t cols,
                                int num_sms, cudaStream_t s, DeviceWeight &dw) {
  const int nb = (int)(cols / 256);
  dw.kind = kind;
  dw.rows = rows;
  dw.cols = cols;
  dw.nb = nb;
  dw.h = choose_tile_height(kind, rows, cols, num_sms);
  dw.ntiles = (int)((rows + dw.h - 1) / dw.h);
  dw.bytes = (uint64_t)dw.ntiles * nb * unit_bytes((int)kind, dw.h);
  const size_t src_bytes = (size_t)rows * nb * packed_block_bytes(kind);
  uint8_t *d_src = nullptr;
  cudaError_t e = cudaMalloc(&dw.units, dw.bytes);
  if (e == cudaSuccess) e = cudaMalloc(&d_src, src_bytes);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_src, host, src_bytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    const long threads = (long)dw.ntiles * nb * dw.h;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    const int r = (int)rows;
#define PRISM_RP(K, HH)                                                               \
  if (kind == K && dw.h == HH)                                                        \
    repack_kernel<K, HH><<<grid, 256, 0, s>>>(d_src, r, nb, dw.ntiles, dw.units);
    PRISM_RP(35, 32) PRISM_RP(35, 16) PRISM_RP(35, 8)
    PRISM_RP(10, 32) PRISM_RP(10, 16) PRISM_RP(10, 8)
#undef PRISM_RP
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (d_src) cudaFree(d_src);
  if (e != cudaSuccess && dw.units) {
    cudaFree(dw.units);
    dw.units = nullptr;
  }
  return e;
}

inline MvWeight mv_weight(const DeviceWeight &w, float *y, const float *residual = nullptr) {
  MvWeight m;
  m.units = w.units;
  m.h = w.h;
  m.ntiles = w.ntiles;
  m.rows = (int)w.rows;
  m.y = y;
  m.residual = residual;
  return m;
}

inline void *matvec_kernel_ptr(uint32_t kind, int epi) {
  if (kind == 35) {
    if (epi == kEpiStore) return reinterpret_cast<void *>(matvec_kernel<35, kEpiStore>);
    if (epi == kEpiArgmax) return reinterpret_cast<void *>(matvec_kernel<35, kEpiArgmax>);
    if (epi == kEpiSwiglu) return reinterpret_cast<void *>(matvec_kernel<35, kEpiSwiglu>);
    return reinterpret_cast<void *>(matvec_kernel<35, kEpiInts>);
  }
  if (epi == kEpiStore) return reinterpret_cast<void *>(matvec_kernel<10, kEpiStore>);
  if (epi == kEpiArgmax) return reinterpret_cast<void *>(matvec_kernel<10, kEpiArgmax>);
  if (epi == kEpiSwiglu) return reinterpret_cast<void *>(matvec_kernel<10, kEpiSwiglu>);
  return reinterpret_cast<void *>(matvec_kernel<10, kEpiInts>);
}

// Allow the largest dynamic shared memory on every projection variant
// (once per device).
inline cudaError_t init_matvec_attributes() {
  for (uint32_t kind : {35u, 10u})
    for (int epi = 0; epi < 4; ++epi) {
      cudaError_t e = cudaFuncSetAttribute(matvec_kernel_ptr(kind, epi),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
      if (e != cudaSuccess) return e;
    }
  return cudaSuccess;
}

// Launch one projection group.  With `pdl`, the launch may begin while the
// previous kernel on the stream finishes (programmatic dependent launch):
// the kernel streams its weights first and waits for the dependency only
// before reading the activation.
// Projection launch policy.  Default (PRISM_B200_MV_PER_SM unset or 0): as
// many one-tile CTAs as fit, up to six per SM, two tiles in flight each --
// measured fastest for batch-1 decode: the integer dots and chains of many
// small CTAs overlap better than fewer CTAs with deeper tile queues, even
// though every CTA rebuilds the Q8_K activation.  PRISM_B200_MV_PER_SM=k
// (1..6) instead aims for k CTAs per SM with all of a CTA's tiles in flight
// (A/B timing).  PRISM_B200_MV_STAGE=1 stages the f32 input in shared memory
// with one round of loads instead of reading it in place (measured neutral;
// the gated-norm prologue always stages).
inline int mv_per_sm() {
  static const int v = [] {
    const char *e = getenv("PRISM_B200_MV_PER_SM");
    const int x = e ? atoi(e) : 0;
    return x < 0 ? 0 : (x > 6 ? 6 : x);
  }();
  return v;
}
inline bool mv_stage() {
  static const bool v = [] {
    const char *e = getenv("PRISM_B200_MV_STAGE");
    return e && e[0] == '1';
  }();
  return v;
}

inline cudaError_t launch_matvec_group(uint32_t kind, int epi, MvArgs a, int num_sms,
                                       cudaStream_t s, bool pdl) {
  int hmax = 8;
  a.tile_start[0] = 0;
  for (int g = 0; g < a.count; ++g) {
    hmax = a.w[g].h > hmax ? a.w[g].h : hmax;
    a.tile_start[g + 1] = a.tile_start[g] + a.w[g].ntiles;
  }
  for (int g = a.count; g < kMaxGroup; ++g) a.tile_start[g + 1] = a.tile_start[a.count];
  const bool pair = epi == kEpiSwiglu;
  if (pair && (a.count != 2 || a.w[0].h != a.w[1].h || a.w[0].rows != a.w[1].rows))
    return cudaErrorInvalidValue;
  const int upt = pair ? 2 * a.nb : a.nb;
  const int unit = unit_bytes((int)kind, hmax);
  const int ntiles = pair ? a.w[0].ntiles : a.tile_start[a.count];
  int grid, smem;
  const int target = mv_per_sm();
  if (target == 0) {
    a.nbuf = 2;
    const int n = a.nb * 256;
    const bool gated = a.prologue == kProGated;  // always staged
    const int stage_n = gated                        ? 2 * n + a.ghd
                        : !mv_stage()                ? 0
                        : a.prologue == kProRmsNorm ? 2 * n
                        : a.prologue == kProF32     ? n
                                                    : 0;
    // resident CTAs per SM (shared memory and registers): a grid beyond
    // them runs in a second wave instead of looping over tiles
    auto resident = [&](int bytes) {
      int per_sm = kSmPerSm / (bytes + 1024);
      if (per_sm > 6) per_sm = 6;
      int occ = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, matvec_kernel_ptr(kind, epi),
                                                        kThreads, (size_t)bytes) == cudaSuccess &&
          occ > 0 && occ < per_sm)
        per_sm = occ;
      return per_sm < 1 ? 1 : per_sm;
    };
    // staging must not cost a resident CTA per SM
    const int plain = MatvecSmem(a.nb, hmax, unit, upt).total();
    const int with = MatvecSmem(a.nb, hmax, unit, upt, 2, stage_n).total();
    a.stage = gated || (stage_n > 0 && with <= kMaxSmem && resident(with) >= resident(plain));
    smem = a.stage ? with : plain;
    if (smem > kMaxSmem) return cudaErrorInvalidValue;
    const int per_sm = resident(smem);
    const long cap = (long)per_sm * num_sms;
    grid = (int)(ntiles < cap ? ntiles : cap);
  } else {
    // about `target` CTAs per SM; one tile per CTA when that barely
    // overfills the SMs.  Each CTA keeps all its tiles in flight when they
    // fit a budget that leaves room for the next kernel's CTA on the SM
    // (its weights stream in under this kernel, programmatic dependent
    // launch), and stages its f32 input in shared memory.
    const long cap = (long)target * num_sms;
    const int per_cta = ntiles <= cap + cap / 4 ? 1 : (int)((ntiles + cap - 1) / cap);
    grid = (ntiles + per_cta - 1) / per_cta;
    const int n = a.nb * 256;
    int stage_n = a.prologue == kProGated ? 2 * n + a.ghd
                  : a.prologue == kProRmsNorm ? 2 * n
                  : a.prologue == kProF32 ? n : 0;
    const int budget = kSmPerSm / (target + 1) - 2048;
    int nbuf = per_cta;
    auto size = [&](int nbf, int sn) { return MatvecSmem(a.nb, hmax, unit, upt, nbf, sn).total(); };
    while (nbuf > 2 && size(nbuf, stage_n) > budget) --nbuf;
    if (size(nbuf, stage_n) > budget && a.prologue != kProGated) stage_n = 0;
    while (nbuf > 1 && size(nbuf, stage_n) > budget) --nbuf;
    smem = size(nbuf, stage_n);
    if (smem > kMaxSmem) return cudaErrorInvalidValue;
    a.nbuf = nbuf;
    a.stage = stage_n > 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void *args[] = {&a};
  return cudaLaunchKernelExC(&cfg, matvec_kernel_ptr(kind, epi), args);
}

// Single-weight projection from prepared Q8_K blocks (or block dots).
inline cudaError_t launch_matvec(const DeviceWeight &w, const void *act, float *y,
                                 int32_t *ints, int32_t *ints2, int epi, unsigned *status,
                                 int num_sms, cudaStream_t s, bool pdl) {
  MvArgs a;
  a.w[0] = mv_weight(w, y);
  a.w[0].ints = ints;
  a.w[0].ints2 = ints2;
  a.count = 1;
  a.nb = w.nb;
  a.prologue = kProQ8K;
  a.in0 = act;
  a.status = status;
  return launch_matvec_group(w.kind, epi, a, num_sms, s, pdl);
}

// Launch configuration with optional programmatic dependent launch; `attr`
// must have room for the caller's extra attributes after index 0.
inline cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     cudaLaunchAttribute *attr, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

inline cudaError_t launch_quantize(const float *x, size_t n, int pinned, void *out,
                                   unsigned *status, cudaStream_t s, bool pdl) {
  int nblocks = (int)(n / 256);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((nblocks * 32 + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  uint8_t *o = static_cast<uint8_t *>(out);
  return cudaLaunchKernelEx(&cfg, q8k_quantize_kernel, x, nblocks, pinned, o, status);
}

}  // namespace prism

struct DeviceBuffer {
  void *ptr = nullptr;
  size_t bytes = 0;
  cudaError_t ensure(size_t need) {
    if (need <= bytes) return cudaSuccess;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    size_t grow = need < 4096 ? 4096 : need;
    cudaError_t e = cudaMalloc(&ptr, grow);
    if (e == cudaSuccess) bytes = grow;
    return e;
  }
  void release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
  }
};

struct prism_b200_weight;

struct prism_b200_executor {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  unsigned *d_status = nullptr;   // device status word(s)
  unsigned *h_status = nullptr;   // pinned mirror
  bool faulted = false;
  bool pdl = true;                // programmatic dependent launch between kernels
  std::string identity;
  std::string last_error;
  DeviceBuffer act, x, y, ints, ints2;
  DeviceBuffer gdn_scratch;       // chunked GDN prefill: per-chunk M, CQ, cum, P
  DeviceBuffer tok_x, tok_act, tok_y;  // multi-token projection: inputs, Q8_K tokens, outputs
  std::set<prism_b200_weight *> weights;

  int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error = buf;
    return code;
  }
};

struct prism_b200_weight {
  prism_b200_executor *ex = nullptr;
  prism::DeviceWeight dw;
};
