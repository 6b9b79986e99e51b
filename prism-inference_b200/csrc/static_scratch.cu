// static_scratch.cu -- the fixed device scratch of
// prism_b200_gdn_prefill_device_noalloc, in a translation unit of its own.
//
// Without relocatable device code each translation unit is a device module
// of its own.  Under CUDA's default lazy module loading a module is loaded
// on a device, and its __device__ variables allocated there, the first time
// one of its functions or variables is used on that device.  No kernel lives
// here, so the array costs its PRISM_B200_GDN_STATIC_SCRATCH_BYTES only on
// devices where the no-allocation prefill has asked for its address (with
// CUDA_MODULE_LOADING=EAGER: on every device the process initialises), and
// it stays allocated there until the context is destroyed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "prism_b200.h"

namespace {

constexpr size_t kFloats = (size_t)PRISM_B200_GDN_STATIC_SCRATCH_BYTES / 4;
static_assert(PRISM_B200_GDN_STATIC_SCRATCH_BYTES % 256 == 0, "scratch size");

__device__ __align__(256) float g_static_gdn_scratch[kFloats];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

CtxGetCurrentFn g_get_current = nullptr;
CtxGetIdFn g_get_id = nullptr;
std::once_flag g_entry_once;

void load_entry_points() {
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_get_id = reinterpret_cast<CtxGetIdFn>(fn);
}

// The driver's process-unique id of the calling thread's current context
// (never reused, unlike the context handle), or 0 when it is unavailable.
unsigned long long current_context_id() {
  std::call_once(g_entry_once, load_entry_points);
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!g_get_current || !g_get_id || g_get_current(&ctx) != CUDA_SUCCESS || !ctx ||
      g_get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

constexpr int kMaxDevices = 64;
struct Entry {
  unsigned long long context;
  float *ptr;
};
std::mutex g_mu;
Entry g_cache[kMaxDevices] = {};

}  // namespace

namespace prism_b200_internal {

// Device address of the fixed scratch in the current context of `device`
// (the caller has made `device` current).  The address is cached per
// context id, so a context destroyed by cudaDeviceReset and created again
// gets the new module's address; without a context id it is looked up on
// every call.  Returns null and sets *err on failure.
__attribute__((visibility("hidden"))) float *static_gdn_scratch(int device, cudaError_t *err) {
  *err = cudaSuccess;
  if (device < 0 || device >= kMaxDevices) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_mu);
  Entry &e = g_cache[device];
  if (ctx && e.context == ctx && e.ptr) return e.ptr;
  void *ptr = nullptr;
  *err = cudaGetSymbolAddress(&ptr, g_static_gdn_scratch);
  if (*err != cudaSuccess) return nullptr;
  e.context = ctx;
  e.ptr = static_cast<float *>(ptr);
  return e.ptr;
}

}  // namespace prism_b200_internal
