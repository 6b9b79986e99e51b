// prism_b200.cu -- C ABI of the quantized projection executor.
//
// Host side of the drop-in boundary declared in include/prism_b200.h.  Each
// entry point validates its arguments before any submission (the
// reference's eligibility-before-submission rule), enqueues sm_100a
// kernels on the executor's stream, and for host-pointer variants waits
// and reads the device status word.  There is no CPU fallback: when a
// kernel cannot run, the call fails.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "executor.cuh"
#include "gdn.cuh"
#include "gdn_op.cuh"
#include "gdn_pinned.cuh"
#include "gemm.cuh"
#include "packed.cuh"
#include "kquant.cuh"

using namespace prism;

namespace {

constexpr size_t kMaxCols = (size_t)kMaxNb * 256;

int status_to_code(unsigned st) {
  if (st & kStatusTimeout) return PRISM_B200_E_TIMEOUT;
  if (st & kStatusNonfinite) return PRISM_B200_E_NONFINITE;
  if (st & kStatusInvalid) return PRISM_B200_E_INVALID;
  return PRISM_B200_OK;
}

int cuda_fail(prism_b200_executor *ex, cudaError_t e, const char *what) {
  return ex->fail(PRISM_B200_E_DEVICE, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what)                                     \
  do {                                                     \
    cudaError_t _e = (call);                               \
    if (_e != cudaSuccess) return cuda_fail(ex, _e, what); \
  } while (0)

int block_bytes(uint32_t kind) {
  if (kind == PRISM_B200_KIND_TQ2_0) return 66;
  if (kind == PRISM_B200_KIND_Q2_K) return 84;
  return 0;
}

bool geometry_ok(const prism_b200_tensor *t) {
  return t && block_bytes(t->kind) != 0 && t->cols > 0 && t->cols % 256 == 0 &&
         t->cols <= kMaxCols && t->rows > 0 && t->rows <= (1ull << 30);
}

// PQ2 / PTQ1 tensors: whole 128-weight blocks (reference src/kernels.rs:
// 88-119 layout, 121-143 dimensions).
bool pq_geometry_ok(const prism_b200_tensor *t) {
  return t && pq_block_bytes(t->kind) != 0 && t->cols > 0 && t->cols % 128 == 0 &&
         t->cols <= kMaxCols && t->rows > 0 && t->rows <= (1ull << 30);
}

// TQ1_0 and Q3_K..Q6_K tensors: whole 256-weight blocks.
bool kquant_geometry_ok(const prism_b200_tensor *t) {
  return t && kquant_block_bytes(t->kind) != 0 && t->cols > 0 && t->cols % 256 == 0 &&
         t->cols <= kMaxCols && t->rows > 0 && t->rows <= (1ull << 30);
}

// Weights kept as uploaded (the reference's block bytes) rather than
// repacked into row tiles: PQ2, PTQ1, TQ1_0, Q3_K..Q6_K.
bool packed_geometry_ok(const prism_b200_tensor *t) {
  return pq_geometry_ok(t) || kquant_geometry_ok(t);
}

// Bytes and weights of one stored block of a packed kind.
int stored_block_bytes(uint32_t kind) {
  return pq_block_bytes(kind) ? pq_block_bytes(kind) : kquant_block_bytes(kind);
}
int stored_block_weights(uint32_t kind) { return pq_block_bytes(kind) ? 128 : 256; }

cudaStream_t pick(prism_b200_executor *ex, void *stream) {
  return stream ? reinterpret_cast<cudaStream_t>(stream) : ex->stream;
}

int check_open(prism_b200_executor *ex) {
  if (!ex) return PRISM_B200_E_INVALID;
  if (ex->faulted)
    return ex->fail(PRISM_B200_E_FAULTED, "executor closed by an earlier failure: %s",
                    ex->last_error.c_str());
  return PRISM_B200_OK;
}

// Wait for the stream and fold the device status into a return code.  Any
// device-side failure closes the executor (no CPU replay).
int finish(prism_b200_executor *ex, cudaStream_t s) {
  CK(cudaMemcpyAsync(ex->h_status, ex->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost, s),
     "status readback");
  CK(cudaStreamSynchronize(s), "stream synchronize");
  unsigned st = *ex->h_status;
  if (st) {
    ex->faulted = true;
    int code = status_to_code(st);
    return ex->fail(code, "device reported status 0x%x", st);
  }
  return PRISM_B200_OK;
}

// A weight of this executor in either layout.
int validate_any_weight(prism_b200_executor *ex, const prism_b200_weight *w) {
  if (!w || w->ex != ex || !w->dw.units)
    return ex->fail(PRISM_B200_E_INVALID, "weight does not belong to this executor");
  return PRISM_B200_OK;
}

// A tiled (TQ2_0 / Q2_K) weight of this executor: every path but the packed
// projections (prism_b200_project, _project_device, _project_q8,
// _project_f32) needs one.
int validate_weight(prism_b200_executor *ex, const prism_b200_weight *w) {
  int st = validate_any_weight(ex, w);
  if (st) return st;
  if (w->dw.packed)
    return ex->fail(PRISM_B200_E_UNSUPPORTED,
                    "PQ2/PTQ1 weights are projected by prism_b200_project, _project_device, "
                    "_project_q8 and _project_f32 only");
  return PRISM_B200_OK;
}

cudaError_t project_on(prism_b200_executor *ex, const prism_b200_weight *w, const void *act,
                       float *y, cudaStream_t s) {
  return launch_matvec(w->dw, act, y, nullptr, nullptr, kEpiStore, ex->d_status, ex->num_sms, s,
                       ex->pdl);
}

// ---- PQ2 / PTQ1 (packed.cuh) ------------------------------------------------

// Whether a packed weight takes Q8_K activations (reference src/kernels.rs:
// 1663-1674): PQ2 with a multiple of 256 columns; PTQ1 and other PQ2 rows
// take Q8_0.
bool packed_q8k(const DeviceWeight &dw) {
  return (dw.kind == 142 && dw.cols % 256 == 0) || kquant_block_bytes(dw.kind) != 0;
}

// Offsets of the fp16 scales of a stored block (every one must be finite).
int block_scale_offsets(uint32_t kind, int *off) {
  switch (kind) {
    case 142: off[0] = 0; return 1;
    case 143: off[0] = 26; return 1;
    case 34: off[0] = 52; return 1;
    case 11: off[0] = 108; return 1;
    case 12: case 13: off[0] = 0; off[1] = 2; return 2;
    case 14: off[0] = 208; return 1;
    default: return 0;
  }
}

int upload_packed(prism_b200_executor *ex, const prism_b200_tensor *t, prism_b200_weight **out) {
  const int bb = stored_block_bytes(t->kind);
  const size_t nb = t->cols / stored_block_weights(t->kind), nblocks = (size_t)t->rows * nb;
  const uint8_t *src = static_cast<const uint8_t *>(t->data);
  int offs[2];
  const int nscales = block_scale_offsets(t->kind, offs);
  for (size_t i = 0; i < nblocks; ++i)
    for (int k = 0; k < nscales; ++k) {
      // every block scale finite (reference scale(), src/kernels.rs:152-154)
      const uint8_t hi = src[i * bb + offs[k] + 1];
      if ((hi & 0x7c) == 0x7c)
        return ex->fail(PRISM_B200_E_NONFINITE, "nonfinite fp16 block scale");
    }
  CK(cudaSetDevice(ex->device), "select device");
  auto *w = new prism_b200_weight();
  w->ex = ex;
  DeviceWeight &dw = w->dw;
  dw.kind = t->kind;
  dw.rows = t->rows;
  dw.cols = t->cols;
  dw.nb = (int)nb;
  dw.h = 0;
  dw.ntiles = 0;
  dw.packed = true;
  dw.bytes = nblocks * (size_t)bb;
  cudaError_t e = cudaMalloc(&dw.units, dw.bytes);
  if (e == cudaSuccess) e = cudaMemcpy(dw.units, src, dw.bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (dw.units) cudaFree(dw.units);
    delete w;
    return cuda_fail(ex, e, "weight upload");
  }
  ex->weights.insert(w);
  *out = w;
  return PRISM_B200_OK;
}

cudaError_t launch_packed(prism_b200_executor *ex, const DeviceWeight &dw, const void *act,
                          bool q8k, int fused, float *y, cudaStream_t s) {
  if (kquant_block_bytes(dw.kind)) {
    KquantArgs k;
    k.w = dw.units;
    k.kind = dw.kind;
    k.rows = (long)dw.rows;
    k.nb = dw.nb;
    k.act = static_cast<const uint8_t *>(act);
    k.y = y;
    k.status = ex->d_status;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)((dw.rows + kKqWarps - 1) / kKqWarps)),
                                        dim3(kKqWarps * 32), 0, s, attr, ex->pdl);
    return cudaLaunchKernelEx(&cfg, kquant_matvec_kernel, k);
  }
  PackedArgs a;
  a.w = dw.units;
  a.kind = dw.kind;
  a.rows = (long)dw.rows;
  a.nb = dw.nb;
  a.act = act;
  a.q8k = q8k ? 1 : 0;
  a.fused = fused ? 1 : 0;
  a.y = y;
  a.status = ex->d_status;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      pdl_config(dim3((unsigned)((dw.rows + kPackedWarps - 1) / kPackedWarps)),
                 dim3(kPackedWarps * 32), 0, s, attr, ex->pdl);
  return cudaLaunchKernelEx(&cfg, packed_matvec_kernel, a);
}

cudaError_t launch_q8_0_quantize(prism_b200_executor *ex, const float *x, size_t n, void *out,
                                 cudaStream_t s) {
  const long nblocks = (long)(n / 32);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)((nblocks * 32 + 255) / 256)), dim3(256), 0,
                                      s, attr, ex->pdl);
  return cudaLaunchKernelEx(&cfg, q8_0_quantize_kernel, x, nblocks, static_cast<Q8Act *>(out),
                            ex->d_status);
}

}  // namespace

extern "C" {

int prism_b200_executor_create(int device, prism_b200_executor **out) {
  if (!out) return PRISM_B200_E_INVALID;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
    return PRISM_B200_E_DEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return PRISM_B200_E_DEVICE;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return PRISM_B200_E_DEVICE;
  if (prop.major < 10) return PRISM_B200_E_UNSUPPORTED;  // sm_100a build only
  auto *ex = new prism_b200_executor();
  ex->device = device;
  ex->num_sms = prop.multiProcessorCount;
  // PRISM_B200_PDL=0 turns programmatic dependent launch off (A/B timing)
  const char *pdl = getenv("PRISM_B200_PDL");
  ex->pdl = !(pdl && pdl[0] == '0');
  if (init_matvec_attributes() != cudaSuccess ||
      cudaStreamCreateWithFlags(&ex->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ex->d_status, 64) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void **>(&ex->h_status), 64, cudaHostAllocDefault) !=
          cudaSuccess ||
      cudaMemset(ex->d_status, 0, 64) != cudaSuccess) {
    prism_b200_executor_destroy(ex);
    return PRISM_B200_E_DEVICE;
  }
  char id[512];
  snprintf(id, sizeof(id), "prism-b200:sm_%d%d:%s:tq2_0+q2_k:q8k-source:tiled-bulk:abi%d",
           prop.major, prop.minor, prop.name, PRISM_B200_ABI_VERSION);
  ex->identity = id;
  *out = ex;
  return PRISM_B200_OK;
}

void prism_b200_executor_destroy(prism_b200_executor *ex) {
  if (!ex) return;
  cudaSetDevice(ex->device);
  if (ex->stream) cudaStreamSynchronize(ex->stream);
  for (auto *w : std::set<prism_b200_weight *>(ex->weights)) prism_b200_weight_release(w);
  ex->act.release();
  ex->x.release();
  ex->y.release();
  ex->ints.release();
  ex->ints2.release();
  ex->gdn_scratch.release();
  ex->tok_x.release();
  ex->tok_act.release();
  ex->tok_y.release();
  if (ex->d_status) cudaFree(ex->d_status);
  if (ex->h_status) cudaFreeHost(ex->h_status);
  if (ex->stream) cudaStreamDestroy(ex->stream);
  delete ex;
}

const char *prism_b200_executor_identity(const prism_b200_executor *ex) {
  return ex ? ex->identity.c_str() : "";
}

size_t prism_b200_executor_last_error(const prism_b200_executor *ex, char *buf, size_t len) {
  if (!ex) return 0;
  if (buf && len) {
    size_t n = ex->last_error.size() < len - 1 ? ex->last_error.size() : len - 1;
    memcpy(buf, ex->last_error.data(), n);
    buf[n] = 0;
  }
  return ex->last_error.size();
}

void *prism_b200_executor_stream(const prism_b200_executor *ex) {
  return ex ? reinterpret_cast<void *>(ex->stream) : nullptr;
}

int prism_b200_executor_sync(prism_b200_executor *ex) {
  if (!ex) return PRISM_B200_E_INVALID;
  cudaSetDevice(ex->device);
  CK(cudaDeviceSynchronize(), "device synchronize");
  return finish(ex, ex->stream);
}

int prism_b200_executor_reset(prism_b200_executor *ex) {
  if (!ex) return PRISM_B200_E_INVALID;
  cudaSetDevice(ex->device);
  CK(cudaDeviceSynchronize(), "device synchronize");
  CK(cudaMemset(ex->d_status, 0, 64), "status reset");
  ex->faulted = false;
  ex->last_error.clear();
  return PRISM_B200_OK;
}

int prism_b200_executor_supports(const prism_b200_executor *ex,
                                 const prism_b200_tensor *tensor) {
  return ex && (geometry_ok(tensor) || packed_geometry_ok(tensor)) ? 1 : 0;
}

int64_t prism_b200_executor_operation_count(const prism_b200_executor *ex,
                                            const prism_b200_tensor *tensor) {
  if (!prism_b200_executor_supports(ex, tensor)) return -1;
  if (packed_geometry_ok(tensor))
    return (int64_t)tensor->rows * (int64_t)(tensor->cols / stored_block_weights(tensor->kind));
  const int h = choose_tile_height(tensor->kind, tensor->rows, tensor->cols, ex->num_sms);
  int64_t tiles = (int64_t)((tensor->rows + h - 1) / h);
  return tiles * (int64_t)(tensor->cols / 256);
}

int prism_b200_weight_upload(prism_b200_executor *ex, const prism_b200_tensor *t,
                             prism_b200_weight **out) {
  int st = check_open(ex);
  if (st) return st;
  if (!out || !t || !t->data) return ex->fail(PRISM_B200_E_INVALID, "null tensor or output");
  *out = nullptr;
  if (packed_geometry_ok(t)) return upload_packed(ex, t, out);
  if (!geometry_ok(t))
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "unsupported kind %u or geometry %llux%llu",
                    t->kind, (unsigned long long)t->cols, (unsigned long long)t->rows);
  const size_t nblocks = (size_t)t->rows * (t->cols / 256);
  const uint8_t *src = static_cast<const uint8_t *>(t->data);
  if (!scales_finite(t->kind, src, nblocks))
    return ex->fail(PRISM_B200_E_NONFINITE, "nonfinite fp16 block scale");
  cudaSetDevice(ex->device);
  auto *w = new prism_b200_weight();
  w->ex = ex;
  cudaError_t e = upload_tiled(src, t->kind, t->rows, t->cols, ex->num_sms, ex->stream, w->dw);
  if (e != cudaSuccess) {
    delete w;
    return cuda_fail(ex, e, "weight upload");
  }
  ex->weights.insert(w);
  *out = w;
  return PRISM_B200_OK;
}

void prism_b200_weight_release(prism_b200_weight *w) {
  if (!w) return;
  if (w->ex) {
    cudaSetDevice(w->ex->device);
    cudaStreamSynchronize(w->ex->stream);
    w->ex->weights.erase(w);
  }
  if (w->dw.units) cudaFree(w->dw.units);
  delete w;
}

uint32_t prism_b200_weight_kind(const prism_b200_weight *w) { return w ? w->dw.kind : 0; }
uint64_t prism_b200_weight_rows(const prism_b200_weight *w) { return w ? w->dw.rows : 0; }
uint64_t prism_b200_weight_cols(const prism_b200_weight *w) { return w ? w->dw.cols : 0; }
uint64_t prism_b200_weight_device_bytes(const prism_b200_weight *w) {
  return w ? w->dw.bytes : 0;
}

int prism_b200_project_device(prism_b200_executor *ex, const prism_b200_weight *w,
                              const void *activation_dev, int fused, float *out_dev,
                              void *stream) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_any_weight(ex, w))) return st;
  if (w->dw.packed && !packed_q8k(w->dw))
    return ex->fail(PRISM_B200_E_UNSUPPORTED,
                    "kind %u with %llu columns takes Q8_0 activations (prism_b200_project_q8)",
                    w->dw.kind, (unsigned long long)w->dw.cols);
  if (!activation_dev || !out_dev) return ex->fail(PRISM_B200_E_INVALID, "null device buffer");
  if (reinterpret_cast<uintptr_t>(activation_dev) % 4)
    return ex->fail(PRISM_B200_E_INVALID, "activation must be 4-byte aligned");
  cudaSetDevice(ex->device);
  if (w->dw.packed)
    CK(launch_packed(ex, w->dw, activation_dev, true, fused, out_dev, pick(ex, stream)),
       "packed matvec launch");
  else
    CK(project_on(ex, w, activation_dev, out_dev, pick(ex, stream)), "matvec launch");
  return PRISM_B200_OK;
}

int prism_b200_project(prism_b200_executor *ex, const prism_b200_weight *w,
                       const prism_b200_q8k_block *activation, int fused, float *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_any_weight(ex, w))) return st;
  if (w->dw.packed && !packed_q8k(w->dw)) {
    if (out) memset(out, 0, w->dw.rows * sizeof(float));
    return ex->fail(PRISM_B200_E_UNSUPPORTED,
                    "kind %u with %llu columns takes Q8_0 activations (prism_b200_project_q8)",
                    w->dw.kind, (unsigned long long)w->dw.cols);
  }
  if (!activation || !out) return ex->fail(PRISM_B200_E_INVALID, "null buffer");
  cudaSetDevice(ex->device);
  const size_t abytes =
      (size_t)(w->dw.packed ? w->dw.cols / 256 : w->dw.nb) * sizeof(prism_b200_q8k_block);
  const size_t ybytes = (size_t)w->dw.rows * sizeof(float);
  CK(ex->act.ensure(abytes), "activation buffer");
  CK(ex->y.ensure(ybytes), "output buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->act.ptr, activation, abytes, cudaMemcpyHostToDevice, s),
     "activation copy");
  if (w->dw.packed)
    CK(launch_packed(ex, w->dw, ex->act.ptr, true, fused, static_cast<float *>(ex->y.ptr), s),
       "packed matvec launch");
  else
    CK(project_on(ex, w, ex->act.ptr, static_cast<float *>(ex->y.ptr), s), "matvec launch");
  CK(cudaMemcpyAsync(out, ex->y.ptr, ybytes, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, ybytes);
  return st;
}

// ---- f32 -> TQ1_0 / TQ2_0 (reference src/kernels/tquants.rs:288-336) --------

static int tq_quantize_check(prism_b200_executor *ex, uint32_t kind, size_t n) {
  if (kind != PRISM_B200_KIND_TQ2_0 && kind != PRISM_B200_KIND_TQ1_0)
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "no quantizer for kind %u", kind);
  if (n == 0 || n % 256 || n / 256 > 0x7fffffffu)
    return ex->fail(PRISM_B200_E_INVALID, "quantizer needs complete 256-value blocks");
  return PRISM_B200_OK;
}

static cudaError_t launch_tq_quantize(prism_b200_executor *ex, uint32_t kind, const float *x,
                                      size_t n, uint8_t *out, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)(n / 256)), dim3(256), 0, s, attr, ex->pdl);
  return cudaLaunchKernelEx(&cfg, tq_quantize_kernel, kind, x, out, ex->d_status);
}

extern "C" int prism_b200_quantize_tq_device(prism_b200_executor *ex, uint32_t kind,
                                             const float *x_dev, size_t n, void *out_dev,
                                             void *stream) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = tq_quantize_check(ex, kind, n))) return st;
  if (!x_dev || !out_dev) return ex->fail(PRISM_B200_E_INVALID, "null device buffer");
  cudaSetDevice(ex->device);
  CK(launch_tq_quantize(ex, kind, x_dev, n, static_cast<uint8_t *>(out_dev), pick(ex, stream)),
     "quantize launch");
  return PRISM_B200_OK;
}

extern "C" int prism_b200_quantize_tq(prism_b200_executor *ex, uint32_t kind, const float *x,
                                      size_t n, void *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = tq_quantize_check(ex, kind, n))) return st;
  if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null buffer");
  const size_t obytes = n / 256 * (kind == PRISM_B200_KIND_TQ2_0 ? 66 : 54);
  cudaSetDevice(ex->device);
  CK(ex->x.ensure(n * sizeof(float)), "input buffer");
  CK(ex->y.ensure(obytes), "output buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->x.ptr, x, n * sizeof(float), cudaMemcpyHostToDevice, s), "input copy");
  CK(launch_tq_quantize(ex, kind, static_cast<const float *>(ex->x.ptr), n,
                        static_cast<uint8_t *>(ex->y.ptr), s),
     "quantize launch");
  if ((st = finish(ex, s))) {
    memset(out, 0, obytes);
    return st;
  }
  CK(cudaMemcpyAsync(out, ex->y.ptr, obytes, cudaMemcpyDeviceToHost, s), "output copy");
  CK(cudaStreamSynchronize(s), "output copy");
  return PRISM_B200_OK;
}

int prism_b200_quantize_q8k_device(prism_b200_executor *ex, const float *x_dev, size_t n,
                                   int pinned, void *out_dev, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  if (!x_dev || !out_dev || n == 0 || n % 256 || n > kMaxCols)
    return ex->fail(PRISM_B200_E_INVALID, "Q8_K activations require a multiple of 256 columns");
  if (reinterpret_cast<uintptr_t>(x_dev) % 16 || reinterpret_cast<uintptr_t>(out_dev) % 4)
    return ex->fail(PRISM_B200_E_INVALID, "misaligned device buffer");
  cudaSetDevice(ex->device);
  CK(launch_quantize(x_dev, n, pinned, out_dev, ex->d_status, pick(ex, stream), ex->pdl),
     "quantize launch");
  return PRISM_B200_OK;
}

int prism_b200_quantize_q8k(prism_b200_executor *ex, const float *x, size_t n, int pinned,
                            prism_b200_q8k_block *out) {
  int st = check_open(ex);
  if (st) return st;
  if (!x || !out || n == 0 || n % 256 || n > kMaxCols)
    return ex->fail(PRISM_B200_E_INVALID, "Q8_K activations require a multiple of 256 columns");
  cudaSetDevice(ex->device);
  const size_t abytes = n / 256 * sizeof(prism_b200_q8k_block);
  CK(ex->x.ensure(n * 4), "input buffer");
  CK(ex->act.ensure(abytes), "activation buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->x.ptr, x, n * 4, cudaMemcpyHostToDevice, s), "input copy");
  CK(launch_quantize(static_cast<float *>(ex->x.ptr), n, pinned, ex->act.ptr, ex->d_status, s,
                     false),
     "quantize");
  CK(cudaMemcpyAsync(out, ex->act.ptr, abytes, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, abytes);
  return st;
}

int prism_b200_project_f32_group(prism_b200_executor *ex, size_t count,
                                 const prism_b200_weight *const *weights, const float *x,
                                 int pinned, float *const *outs) {
  int st = check_open(ex);
  if (st) return st;
  if (!count || !weights || !x || !outs) return ex->fail(PRISM_B200_E_INVALID, "empty group");
  if ((st = validate_weight(ex, weights[0]))) return st;
  const uint64_t cols = weights[0]->dw.cols;
  size_t total_rows = 0;
  for (size_t i = 0; i < count; ++i) {
    if ((st = validate_weight(ex, weights[i]))) return st;
    if (weights[i]->dw.cols != cols)
      return ex->fail(PRISM_B200_E_INVALID, "mismatched projection group columns");
    if (!outs[i]) return ex->fail(PRISM_B200_E_INVALID, "null output");
    total_rows += weights[i]->dw.rows;
  }
  cudaSetDevice(ex->device);
  const size_t n = cols;
  const size_t abytes = n / 256 * sizeof(prism_b200_q8k_block);
  CK(ex->x.ensure(n * 4), "input buffer");
  CK(ex->act.ensure(abytes), "activation buffer");
  CK(ex->y.ensure(total_rows * 4), "output buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->x.ptr, x, n * 4, cudaMemcpyHostToDevice, s), "input copy");
  CK(launch_quantize(static_cast<float *>(ex->x.ptr), n, pinned, ex->act.ptr, ex->d_status, s,
                     false),
     "quantize");
  size_t off = 0;
  for (size_t i = 0; i < count; ++i) {
    float *y = static_cast<float *>(ex->y.ptr) + off;
    CK(project_on(ex, weights[i], ex->act.ptr, y, s), "matvec launch");
    off += weights[i]->dw.rows;
  }
  off = 0;
  for (size_t i = 0; i < count; ++i) {
    float *y = static_cast<float *>(ex->y.ptr) + off;
    CK(cudaMemcpyAsync(outs[i], y, weights[i]->dw.rows * 4, cudaMemcpyDeviceToHost, s),
       "output copy");
    off += weights[i]->dw.rows;
  }
  st = finish(ex, s);
  if (st)
    for (size_t i = 0; i < count; ++i) memset(outs[i], 0, weights[i]->dw.rows * 4);
  return st;
}

int prism_b200_project_f32(prism_b200_executor *ex, const prism_b200_weight *w, const float *x,
                           int pinned, float *out) {
  if (ex && w && w->ex == ex && w->dw.packed) {
    // PQ2 / PTQ1: quantized by the tensor's activation contract, unfused
    int st = check_open(ex);
    if (st) return st;
    if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null buffer");
    if (pinned)
      return ex->fail(PRISM_B200_E_UNSUPPORTED, "pinned accumulation of kind %u", w->dw.kind);
    const DeviceWeight &dw = w->dw;
    const bool q8k = packed_q8k(dw);
    const size_t n = dw.cols;
    const size_t abytes = q8k ? n / 256 * sizeof(prism_b200_q8k_block) : n / 32 * sizeof(Q8Act);
    const size_t ybytes = (size_t)dw.rows * sizeof(float);
    CK(cudaSetDevice(ex->device), "select device");
    CK(ex->x.ensure(n * sizeof(float)), "input buffer");
    CK(ex->act.ensure(abytes), "activation buffer");
    CK(ex->y.ensure(ybytes), "output buffer");
    cudaStream_t s = ex->stream;
    float *xd = static_cast<float *>(ex->x.ptr);
    CK(cudaMemcpyAsync(xd, x, n * sizeof(float), cudaMemcpyHostToDevice, s), "input copy");
    if (q8k)
      CK(launch_quantize(xd, n, 0, ex->act.ptr, ex->d_status, s, ex->pdl), "quantize launch");
    else
      CK(launch_q8_0_quantize(ex, xd, n, ex->act.ptr, s), "quantize launch");
    CK(launch_packed(ex, dw, ex->act.ptr, q8k, 0, static_cast<float *>(ex->y.ptr), s),
       "packed matvec launch");
    CK(cudaMemcpyAsync(out, ex->y.ptr, ybytes, cudaMemcpyDeviceToHost, s), "output copy");
    st = finish(ex, s);
    if (st) memset(out, 0, ybytes);
    return st;
  }
  const prism_b200_weight *ws[1] = {w};
  float *os[1] = {out};
  return prism_b200_project_f32_group(ex, 1, ws, x, pinned, os);
}

int prism_b200_project_f32_tokens_device(prism_b200_executor *ex, const prism_b200_weight *w,
                                         size_t tokens, const float *x_dev, int pinned,
                                         float *out_dev, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, w))) return st;
  if (!tokens) return PRISM_B200_OK;
  if (!x_dev || !out_dev) return ex->fail(PRISM_B200_E_INVALID, "null device buffer");
  if (reinterpret_cast<uintptr_t>(x_dev) % 16 || reinterpret_cast<uintptr_t>(out_dev) % 4)
    return ex->fail(PRISM_B200_E_INVALID, "misaligned token buffers");
  if (tokens > (size_t)kMaxTokens)
    return ex->fail(PRISM_B200_E_INVALID, "at most %d tokens per call", kMaxTokens);
  CK(cudaSetDevice(ex->device), "select device");
  const DeviceWeight &dw = w->dw;
  const size_t M = tokens, nb = dw.nb;
  // Q8_K tokens, tile-major over 128-token tiles (gemm.cuh token_q8k_carve)
  CK(ex->tok_act.ensure(token_q8k_bytes(M, (int)nb)), "token activation buffer");
  const TokenQ8K t = token_q8k_carve(ex->tok_act.ptr, M, (int)nb);
  cudaStream_t s = pick(ex, stream);
  CK(launch_token_gemm(dw, x_dev, M, pinned, t, out_dev, ex->d_status, s, ex->pdl),
     "token projection launch");
  return PRISM_B200_OK;
}

int prism_b200_project_f32_tokens(prism_b200_executor *ex, const prism_b200_weight *w,
                                  size_t tokens, const float *x, int pinned, float *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, w))) return st;
  if (!tokens) return PRISM_B200_OK;
  if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null token buffer");
  if (tokens > (size_t)kMaxTokens)
    return ex->fail(PRISM_B200_E_INVALID, "at most %d tokens per call", kMaxTokens);
  CK(cudaSetDevice(ex->device), "select device");
  const size_t xin = tokens * w->dw.cols * 4, yout = tokens * w->dw.rows * 4;
  CK(ex->tok_x.ensure(xin), "token input buffer");
  CK(ex->tok_y.ensure(yout), "token output buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->tok_x.ptr, x, xin, cudaMemcpyHostToDevice, s), "input copy");
  if ((st = prism_b200_project_f32_tokens_device(ex, w, tokens,
                                                 static_cast<float *>(ex->tok_x.ptr), pinned,
                                                 static_cast<float *>(ex->tok_y.ptr), s)))
    return st;
  CK(cudaMemcpyAsync(out, ex->tok_y.ptr, yout, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, yout);
  return st;
}

int prism_b200_block_dots(prism_b200_executor *ex, const prism_b200_weight *w,
                          const prism_b200_q8k_block *activation, int32_t *ints,
                          int32_t *ints2) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, w))) return st;
  if (!activation || !ints || (w->dw.kind == PRISM_B200_KIND_Q2_K && !ints2))
    return ex->fail(PRISM_B200_E_INVALID, "null buffer");
  cudaSetDevice(ex->device);
  const size_t abytes = (size_t)w->dw.nb * sizeof(prism_b200_q8k_block);
  const size_t ibytes = (size_t)w->dw.rows * w->dw.nb * 4;
  CK(ex->act.ensure(abytes), "activation buffer");
  CK(ex->ints.ensure(ibytes), "ints buffer");
  CK(ex->ints2.ensure(ibytes), "ints buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->act.ptr, activation, abytes, cudaMemcpyHostToDevice, s),
     "activation copy");
  CK(launch_matvec(w->dw, ex->act.ptr, nullptr, static_cast<int32_t *>(ex->ints.ptr),
                   static_cast<int32_t *>(ex->ints2.ptr), kEpiInts, ex->d_status, ex->num_sms, s,
                   false),
     "block dots launch");
  CK(cudaMemcpyAsync(ints, ex->ints.ptr, ibytes, cudaMemcpyDeviceToHost, s), "ints copy");
  if (w->dw.kind == PRISM_B200_KIND_Q2_K)
    CK(cudaMemcpyAsync(ints2, ex->ints2.ptr, ibytes, cudaMemcpyDeviceToHost, s), "ints copy");
  return finish(ex, s);
}

// ---- Gated DeltaNet recurrence ---------------------------------------------

static int gdn_check(prism_b200_executor *ex, int batch, int tokens, int heads, int key_heads,
                     int d, const void *const *ptrs, int n) {
  if (batch <= 0 || tokens <= 0 || heads <= 0 || key_heads <= 0 || heads % key_heads ||
      batch > 65535 || heads > 65535)
    return ex->fail(PRISM_B200_E_INVALID, "invalid GDN geometry");
  if (d != kGdnD) return ex->fail(PRISM_B200_E_UNSUPPORTED, "GDN head width must be 128");
  for (int i = 0; i < n; ++i)
    if (!ptrs[i] || reinterpret_cast<uintptr_t>(ptrs[i]) % 16)
      return ex->fail(PRISM_B200_E_INVALID, "GDN buffers must be 16-byte aligned device memory");
  return PRISM_B200_OK;
}

extern "C" int prism_b200_gdn_decode_device(prism_b200_executor *ex, int batch, int heads,
                                            int key_heads, int d, float *state, const float *q,
                                            const float *k, const float *v, const float *decay,
                                            const float *beta, float *out, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  const void *ptrs[] = {state, q, k, v, out};
  if ((st = gdn_check(ex, batch, 1, heads, key_heads, d, ptrs, 5))) return st;
  if (!decay || !beta) return ex->fail(PRISM_B200_E_INVALID, "null gate buffer");
  cudaSetDevice(ex->device);
  GdnBatchArgs a;
  a.batch = batch;
  a.T = 1;
  a.heads = heads;
  a.key_heads = key_heads;
  a.state = state;
  a.q = q;
  a.k = k;
  a.v = v;
  a.decay = decay;
  a.beta = beta;
  a.out = out;
  a.status = ex->d_status;
  // split each head's 128 rows so that the grid covers every SM twice and a
  // warp holds at most kGdnRowBatch rows (one round of loads)
  int split = 128 / (kGdnStepThreads / 32 * kGdnRowBatch);
  while (split < 16 && (long)batch * heads * split < 2L * ex->num_sms) split *= 2;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(split, heads, batch), dim3(kGdnStepThreads), 0,
                                      pick(ex, stream), attr, ex->pdl);
  CK(cudaLaunchKernelEx(&cfg, gdn_step_kernel, a), "GDN decode launch");
  return PRISM_B200_OK;
}

extern "C" int prism_b200_gdn_prefill_device(prism_b200_executor *ex, int batch, int tokens,
                                             int heads, int key_heads, int d, int chunk,
                                             float *state, const float *q, const float *k,
                                             const float *v, const float *decay,
                                             const float *beta, float *out, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  const void *ptrs[] = {state, q, k, v, out};
  if ((st = gdn_check(ex, batch, tokens, heads, key_heads, d, ptrs, 5))) return st;
  if (!decay || !beta) return ex->fail(PRISM_B200_E_INVALID, "null gate buffer");
  if (chunk < 1 || chunk > kChunk)
    return ex->fail(PRISM_B200_E_INVALID, "GDN chunk must be 1..%d tokens", kChunk);
  cudaSetDevice(ex->device);
  GdnPrefillArgs p;
  p.g.batch = batch;
  p.g.T = tokens;
  p.g.heads = heads;
  p.g.key_heads = key_heads;
  p.g.state = state;
  p.g.q = q;
  p.g.k = k;
  p.g.v = v;
  p.g.decay = decay;
  p.g.beta = beta;
  p.g.out = out;
  p.g.status = ex->d_status;
  p.chunk = chunk;
  p.nchunks = (tokens + chunk - 1) / chunk;
  const size_t scratch = (size_t)batch * heads * p.nchunks * kChunkScratch * sizeof(float);
  CK(ex->gdn_scratch.ensure(scratch), "GDN scratch");
  p.scratch = static_cast<float *>(ex->gdn_scratch.ptr);
  cudaStream_t s = pick(ex, stream);
  cudaLaunchAttribute attr[1];
  const size_t prep_smem = gdn_prep_smem();
  CK(cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)prep_smem),
     "GDN prep attribute");
  cudaLaunchConfig_t cfg = pdl_config(dim3(p.nchunks, heads, batch), dim3(kPrepThreads),
                                      prep_smem, s, attr, ex->pdl);
  CK(cudaLaunchKernelEx(&cfg, gdn_chunk_prep_kernel, p), "GDN prep launch");
  {
    const size_t smem = gdn_chunk_scan_smem();
    CK(cudaFuncSetAttribute(gdn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)smem),
       "GDN scan attribute");
    cfg = pdl_config(dim3(kGdnD / kScanR, heads, batch), dim3(kScanThreads), smem, s, attr,
                     ex->pdl);
    CK(cudaLaunchKernelEx(&cfg, gdn_chunk_scan_kernel, p), "GDN scan launch");
  }
  return PRISM_B200_OK;
}

extern "C" int prism_b200_gdn_prefill_pinned_device(prism_b200_executor *ex, int batch,
                                                    int tokens, int heads, int key_heads, int d,
                                                    float *state, const float *q, const float *k,
                                                    const float *v, const float *decay,
                                                    const float *beta, float *out, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  const void *ptrs[] = {state, q, k, v, out};
  if ((st = gdn_check(ex, batch, tokens, heads, key_heads, d, ptrs, 5))) return st;
  if (!decay || !beta) return ex->fail(PRISM_B200_E_INVALID, "null gate buffer");
  cudaSetDevice(ex->device);
  GdnBatchArgs a;
  a.batch = batch;
  a.T = tokens;
  a.heads = heads;
  a.key_heads = key_heads;
  a.state = state;
  a.q = q;
  a.k = k;
  a.v = v;
  a.decay = decay;
  a.beta = beta;
  a.out = out;
  a.status = ex->d_status;
  cudaStream_t s = pick(ex, stream);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(heads, batch), dim3(kPinnedD), 0, s, attr, ex->pdl);
  CK(cudaLaunchKernelEx(&cfg, gdn_pinned_kernel, a), "pinned GDN launch");
  return PRISM_B200_OK;
}

}  // extern "C"

// ---- GDN prefill with no device allocation ---------------------------------
// Some hosts cannot let a library allocate device memory behind their back:
// a serving process that reserved all of HBM up front for weights and KV
// pages has none left to give, and a decode loop with a latency budget
// cannot absorb the device-wide synchronisation that cudaMalloc implies.
// ---- the batched gated-delta op with snapshots / replay (gdn_op.cuh) ---------

extern "C" size_t prism_b200_gdn_delta_values_outputs(const prism_b200_gdn_op *op) {
  if (!op) return 0;
  return gdn_op_outputs(op->width, op->heads, op->tokens, op->sequences, op->snapshots,
                        op->replay != 0);
}

extern "C" int prism_b200_gdn_delta_values_device(
    prism_b200_executor *ex, const prism_b200_gdn_op *op, const float *q, const float *k,
    const float *v, const float *gate, const float *beta, const float *table,
    const int32_t *rows, const float *bias, const float *weight, const float *records,
    const int32_t *control, float *out, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  if (!op) return ex->fail(PRISM_B200_E_INVALID, "null op");
  const prism_b200_gdn_op &o = *op;
  if (o.snapshots == 0 || (o.replay && o.snapshots < 2) || (o.replay && o.raw))
    return ex->fail(PRISM_B200_E_INVALID, "snapshot count, or raw gates with replay");
  if (o.width == 0 || o.heads == 0 || o.sequences == 0 || (o.replay && o.tokens == 0) ||
      o.q_heads == 0 || o.k_heads == 0 || o.q_sequences == 0 || o.k_sequences == 0 ||
      o.sequences % o.q_sequences || o.sequences % o.k_sequences ||
      (o.gate_width != 1 && o.gate_width != o.width) || o.state_rows == 0 ||
      o.heads > 65535u || o.sequences > 65535u)
    return ex->fail(PRISM_B200_E_INVALID, "gated-delta op geometry");
  if (o.width > (uint32_t)kGdnOpMaxWidth)
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "state width %u above %d", o.width,
                    kGdnOpMaxWidth);
  if (!q || !k || !v || !gate || !beta || !table || !out ||
      (o.raw && (!bias || !weight)) || (o.replay && (!records || !control || o.record_banks == 0)))
    return ex->fail(PRISM_B200_E_INVALID, "null input");
  GdnOpArgs a;
  a.W = (int)o.width;
  a.H = (int)o.heads;
  a.T = (int)o.tokens;
  a.S = (int)o.sequences;
  a.qh = (int)o.q_heads;
  a.kh = (int)o.k_heads;
  a.qs = (int)o.q_sequences;
  a.ks = (int)o.k_sequences;
  a.gw = (int)o.gate_width;
  a.snaps = (int)o.snapshots;
  a.raw = o.raw ? 1 : 0;
  a.replay = o.replay ? 1 : 0;
  a.state_rows = (int)o.state_rows;
  a.banks = (int)o.record_banks;
  a.bank_elems = (long)o.record_bank_elems;
  a.records_len = (long)o.records_len;
  a.q = q;
  a.k = k;
  a.v = v;
  a.gate = gate;
  a.beta = beta;
  a.table = table;
  a.rows = o.replay ? nullptr : rows;
  a.bias = bias;
  a.weight = weight;
  a.records = records;
  a.control = control;
  a.out = out;
  a.status = ex->d_status;
  const size_t smem = ((size_t)o.width * (o.width + 1) + 3 * (size_t)o.width) * 4;
  cudaSetDevice(ex->device);
  CK(cudaFuncSetAttribute(gdn_op_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
     "gated-delta op attribute");
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(o.heads, o.sequences), dim3(kGdnOpMaxWidth), smem,
                                      pick(ex, stream), attr, ex->pdl);
  CK(cudaLaunchKernelEx(&cfg, gdn_op_kernel, a), "gated-delta op launch");
  return PRISM_B200_OK;
}

// This variant of prism_b200_gdn_prefill_device keeps its chunk scratch in
// a fixed module-scope array (static_scratch.cu) instead of the executor's
// growable buffer.  The prep kernel writes every scratch element that the
// scan kernel reads, so nothing has to start at zero.  The array is shared
// by every caller on a device: two calls whose kernels overlap in time
// (different streams, or different executors on one device) race on it.
namespace prism_b200_internal {
float *static_gdn_scratch(int device, cudaError_t *err);
}
namespace {
constexpr size_t kStaticGdnScratchFloats = (size_t)PRISM_B200_GDN_STATIC_SCRATCH_BYTES / 4;
}  // namespace

extern "C" int prism_b200_gdn_prefill_device_noalloc(prism_b200_executor *ex, int batch,
                                                     int tokens, int heads, int key_heads, int d,
                                                     int chunk, float *state, const float *q,
                                                     const float *k, const float *v,
                                                     const float *decay, const float *beta,
                                                     float *out, void *stream) {
  int st = check_open(ex);
  if (st) return st;
  const void *ptrs[] = {state, q, k, v, out};
  if ((st = gdn_check(ex, batch, tokens, heads, key_heads, d, ptrs, 5))) return st;
  if (!decay || !beta) return ex->fail(PRISM_B200_E_INVALID, "null gate buffer");
  if (chunk < 1 || chunk > kChunk)
    return ex->fail(PRISM_B200_E_INVALID, "GDN chunk must be 1..%d tokens", kChunk);
  const long nchunks = (tokens + chunk - 1) / chunk;
  const size_t need = (size_t)batch * heads * nchunks * kChunkScratch;
  if (need > kStaticGdnScratchFloats)
    return ex->fail(PRISM_B200_E_INVALID,
                    "GDN no-alloc prefill needs %zu scratch bytes (batch %d x heads %d x %ld "
                    "chunks x %d B); the fixed scratch holds %zu",
                    need * 4, batch, heads, nchunks, kChunkScratch * 4,
                    (size_t)PRISM_B200_GDN_STATIC_SCRATCH_BYTES);
  CK(cudaSetDevice(ex->device), "select device");
  cudaError_t e;
  float *scratch = prism_b200_internal::static_gdn_scratch(ex->device, &e);
  if (!scratch) return cuda_fail(ex, e, "GDN fixed scratch address");
  GdnPrefillArgs p;
  p.g.batch = batch;
  p.g.T = tokens;
  p.g.heads = heads;
  p.g.key_heads = key_heads;
  p.g.state = state;
  p.g.q = q;
  p.g.k = k;
  p.g.v = v;
  p.g.decay = decay;
  p.g.beta = beta;
  p.g.out = out;
  p.g.status = ex->d_status;
  p.chunk = chunk;
  p.nchunks = (int)nchunks;
  p.scratch = scratch;
  cudaStream_t s = pick(ex, stream);
  cudaLaunchAttribute attr[1];
  const size_t prep_smem = gdn_prep_smem();
  CK(cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)prep_smem),
     "GDN prep attribute");
  cudaLaunchConfig_t cfg = pdl_config(dim3(p.nchunks, heads, batch), dim3(kPrepThreads),
                                      prep_smem, s, attr, ex->pdl);
  CK(cudaLaunchKernelEx(&cfg, gdn_chunk_prep_kernel, p), "GDN prep launch");
  {
    const size_t smem = gdn_chunk_scan_smem();
    CK(cudaFuncSetAttribute(gdn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)smem),
       "GDN scan attribute");
    cfg = pdl_config(dim3(kGdnD / kScanR, heads, batch), dim3(kScanThreads), smem, s, attr,
                     ex->pdl);
    CK(cudaLaunchKernelEx(&cfg, gdn_chunk_scan_kernel, p), "GDN scan launch");
  }
  return PRISM_B200_OK;
}

// The model entry points share this translation unit's kernels and helpers.
#include "model.cuh"
#include "checkpoint.cuh"
#include "gguf.cuh"
#include "batch.cuh"
#include "prefill.cuh"
#include "tp_ffn.cuh"
#include "peak.cuh"
#include "seam.cuh"
