// executor.cuh -- host-side executor state shared by the C ABI translation
// units.  Not part of the public ABI.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <set>
#include <string>

#include <cuda_runtime.h>

#include "../../include/prism_b200.h"

struct prism_b200_weight;

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

struct prism_b200_executor {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  unsigned *d_status = nullptr;   // device status word(s)
  unsigned *h_status = nullptr;   // pinned mirror
  bool faulted = false;
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
  uint32_t kind = 0;
  uint64_t rows = 0, cols = 0;
  int nb = 0, ntiles = 0;
  uint8_t *d_units = nullptr;
  float *d_partial = nullptr;     // ntiles*nb*32 floats
  unsigned *d_cnt = nullptr;      // ntiles counters
  uint64_t unit_bytes = 0;
  uint64_t device_bytes = 0;
};
