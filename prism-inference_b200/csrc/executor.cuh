// executor.cuh -- host-side executor state and kernel launch helpers shared
// by the C ABI translation units.  Not part of the public ABI.
#pragma once

#include <cstdarg>
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
  int grid = 0;         // persistent CTAs per launch
  int smem = 0;         // dynamic shared memory per CTA
};

// Tile height: the largest of 32/16/8 rows that still gives every SM a tile
// (tiles of 32 rows use one lane per row; 16 and 8 split a row's four
// 16-byte chunks over 2 or 4 lanes).
// The double-buffered tile must also fit the 227 KB shared-memory budget.
constexpr int kMaxSmem = 232448;
inline int choose_tile_height(uint32_t kind, uint64_t rows, uint64_t cols, int num_sms) {
  int h = 8;
  if ((rows + 31) / 32 >= (uint64_t)2 * num_sms) h = 32;
  else if ((rows + 15) / 16 >= (uint64_t)num_sms) h = 16;
  const int nb = (int)(cols / 256);
  while (h > 8 && MatvecSmem(nb, h, unit_bytes((int)kind, h)).total() > kMaxSmem) h /= 2;
  return h;
}

template <int KIND, int H, int MODE>
inline void *matvec_fn() {
  return reinterpret_cast<void *>(matvec_kernel<KIND, H, MODE, true>);
}

inline void *matvec_kernel_ptr(uint32_t kind, int h, int mode) {
#define PRISM_MV(K, HH)                                                            \
  if (kind == K && h == HH) return mode == kModeOutput ? matvec_fn<K, HH, kModeOutput>() \
                                                       : matvec_fn<K, HH, kModeInts>();
  PRISM_MV(35, 32) PRISM_MV(35, 16) PRISM_MV(35, 8)
  PRISM_MV(10, 32) PRISM_MV(10, 16) PRISM_MV(10, 8)
#undef PRISM_MV
  return nullptr;
}

// Configure grid and shared memory once per weight (at upload).
inline cudaError_t configure_weight(DeviceWeight &w, int num_sms) {
  const int unit = unit_bytes((int)w.kind, w.h);
  const MatvecSmem L(w.nb, w.h, unit);
  w.smem = L.total();
  int max_blocks = 0;
  for (int mode = 0; mode < 2; ++mode) {
    void *fn = matvec_kernel_ptr(w.kind, w.h, mode);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, w.smem);
    if (e != cudaSuccess) return e;
    if (mode == 0) {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&max_blocks, fn, kThreads, w.smem);
      if (e != cudaSuccess) return e;
    }
  }
  if (max_blocks < 1) return cudaErrorInvalidConfiguration;
  long cap = (long)max_blocks * num_sms;
  w.grid = (int)(w.ntiles < cap ? w.ntiles : cap);
  return cudaSuccess;
}

// Launch one projection.  With `pdl`, the launch may begin while the
// previous kernel on the stream finishes (programmatic dependent launch):
// the kernel streams its weights first and waits for the dependency only
// before reading the activation.
inline cudaError_t launch_matvec(const DeviceWeight &w, const void *act, float *y,
                                 int32_t *ints, int32_t *ints2, int mode, unsigned *status,
                                 cudaStream_t s, bool pdl) {
  MatvecArgs a;
  a.w = w.units;
  a.act = static_cast<const uint8_t *>(act);
  a.nb = w.nb;
  a.ntiles = w.ntiles;
  a.rows = (int)w.rows;
  a.y = y;
  a.ints = ints;
  a.ints2 = ints2;
  a.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)w.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)w.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void *args[] = {&a};
  return cudaLaunchKernelExC(&cfg, matvec_kernel_ptr(w.kind, w.h, mode), args);
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
