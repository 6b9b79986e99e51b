// tp_ffn.cuh -- the FFN chain over a tile of tokens, on one GPU or
// tensor-parallel over several.
//
// The reference's full intra-layer FFN chain over token activations
// (src/kernels/projection.rs:261-350 project_f32_ffn_chain_tokens: ffn_gate,
// ffn_up, SwiGLU, ffn_down, optional residual) as one resident object:
//   out[m] = residual[m] + down(Q8_K(up(Q8_K(x_m)) * silu(gate(Q8_K(x_m)))))
// with every projection on the tensor cores (gemm.cuh) and the reference's
// per-row binary32 chains; on one GPU the result is the sequential chain's,
// bit for bit.
//
// Tensor-parallel over N ranks (one process and GPU each): rank r holds
// gate/up rows [r*F/N, (r+1)*F/N) (column parallel) and the matching input
// blocks of ffn_down (row parallel).  Its down GEMM's epilogue stores the
// partial [M][H] into receive slot r of every rank's exchange buffer and
// counts the delivered values on that rank's arrival counter; each rank's
// reduce kernel waits (bounded) for all N partials, adds them in rank order
// and adds the residual -- an all-reduce fused into the producing GEMM and
// the consuming kernel, over plain peer stores through NVLink.  The rank
// sums round differently from one sequential chain (a relative difference
// of a few binary32 ulps of the partials).
#pragma once

#include "batch.cuh"

struct prism_b200_ffn {
  prism_b200_executor *ex = nullptr;
  int rank = 0, size = 1;
  size_t max_tokens = 0;
  int H = 0, F = 0, Fl = 0;               // hidden, FFN width, this rank's FFN width
  prism::DeviceWeight gate, up, down;     // this rank's slices (views at size 1)
  void *tok = nullptr;                    // Q8_K tokens of the widest input
  float *g = nullptr, *u = nullptr;       // [M][Fl]
  prism::TpExchange x;                    // all-reduce slots (size > 1)
  unsigned long long *zero = nullptr;     // device 0: the waits' step count
  uint64_t calls = 0;                     // calls completed on this rank
  unsigned long long delivered = 0;       // values every rank's counter has received
  std::vector<void *> allocs;
};

namespace prism {

// out[row] = residual[row] + (slot 0 + slot 1 + ... in rank order), after
// every rank's partial of this call has arrived.  grid (M), 256 threads.
__global__ void __launch_bounds__(256) tp_ffn_reduce_kernel(const float *slots, int ranks, int M,
                                                            int n, TpWait w,
                                                            const float *residual, float *out,
                                                            unsigned *status) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = tp_wait(w, status);
  __syncthreads();
  if (!ok) return;
  const long row = blockIdx.x;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float s = __ldcg(slots + row * n + i);
    for (int p = 1; p < ranks; ++p) s = __fadd_rn(s, __ldcg(slots + ((long)p * M + row) * n + i));
    const float v = residual ? __fadd_rn(residual[row * n + i], s) : s;
    if (!is_finite_f(v)) report(status, kStatusNonfinite);
    out[row * n + i] = v;
  }
}

}  // namespace prism

int prism_b200_ffn_create(prism_b200_executor *ex, const prism_b200_weight *gate,
                          const prism_b200_weight *up, const prism_b200_weight *down,
                          uint32_t max_tokens, uint32_t tp_rank, uint32_t tp_size,
                          prism_b200_ffn **out) {
  using namespace prism;
  if (!ex || !out) return PRISM_B200_E_INVALID;
  *out = nullptr;
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, gate)) || (st = validate_weight(ex, up)) ||
      (st = validate_weight(ex, down)))
    return st;
  const DeviceWeight &G = gate->dw, &U = up->dw, &D = down->dw;
  if (G.kind != U.kind || G.kind != D.kind || G.rows != U.rows || G.cols != U.cols ||
      D.rows != G.cols || D.cols != G.rows)
    return ex->fail(PRISM_B200_E_INVALID,
                    "FFN chain wants gate and up [F][H] and down [H][F] of one kind");
  if (max_tokens == 0 || max_tokens > (uint32_t)kMaxTokens)
    return ex->fail(PRISM_B200_E_INVALID, "between 1 and %d tokens per call", kMaxTokens);
  if (tp_size < 1 || tp_size > (uint32_t)kMaxTp || tp_rank >= tp_size)
    return ex->fail(PRISM_B200_E_INVALID, "rank %u of %u", tp_rank, tp_size);
  const int F = (int)G.rows, H = (int)G.cols;
  if (F % (256 * (int)tp_size))
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "FFN width %d does not split into %u x 256-column "
                    "blocks", F, tp_size);
  CK(cudaSetDevice(ex->device), "select device");
  auto *f = new prism_b200_ffn;
  f->ex = ex;
  f->rank = (int)tp_rank;
  f->size = (int)tp_size;
  f->max_tokens = max_tokens;
  f->H = H;
  f->F = F;
  f->Fl = F / (int)tp_size;
  cudaStream_t s = ex->stream;
  cudaError_t e = cudaSuccess;
  if (tp_size == 1) {
    f->gate = G;
    f->up = U;
    f->down = D;
  } else {
    const int r0 = f->rank * f->Fl;
    const std::vector<int> frows = tp_rows({{r0, r0 + f->Fl}});
    std::vector<int> hrows(H);
    for (int i = 0; i < H; ++i) hrows[i] = i;
    e = tp_gather_weight(G, frows, 0, G.nb, ex->num_sms, f->allocs, s, f->gate);
    if (e == cudaSuccess) e = tp_gather_weight(U, frows, 0, U.nb, ex->num_sms, f->allocs, s, f->up);
    if (e == cudaSuccess)
      e = tp_gather_weight(D, hrows, r0 / 256, f->Fl / 256, ex->num_sms, f->allocs, s, f->down);
  }
  auto A = [&](void **p, size_t bytes) {
    if (e != cudaSuccess) return;
    e = cudaMalloc(p, bytes < 16 ? 16 : bytes);
    if (e == cudaSuccess) f->allocs.push_back(*p);
  };
  const int widest = std::max(H, f->Fl) / 256;
  A(&f->tok, token_q8k_bytes(max_tokens, widest));
  A(reinterpret_cast<void **>(&f->g), (size_t)max_tokens * f->Fl * 4);
  A(reinterpret_cast<void **>(&f->u), (size_t)max_tokens * f->Fl * 4);
  if (tp_size > 1) {
    f->x.layout(kTpAllReduce, f->size, (int)max_tokens, H, 0);
    void *xb = nullptr;
    A(&xb, f->x.bytes);
    if (e == cudaSuccess) e = cudaMemset(xb, 0, f->x.bytes);
    f->x.base = static_cast<uint8_t *>(xb);
    A(reinterpret_cast<void **>(&f->zero), 16);
    if (e == cudaSuccess) e = cudaMemset(f->zero, 0, 16);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    prism_b200_ffn_destroy(f);
    return cuda_fail(ex, e, "FFN chain setup");
  }
  *out = f;
  return PRISM_B200_OK;
}

void prism_b200_ffn_destroy(prism_b200_ffn *f) {
  if (!f) return;
  cudaSetDevice(f->ex->device);
  cudaStreamSynchronize(f->ex->stream);
  for (int p = 0; p < prism::kMaxTp; ++p)
    if (f->x.opened[p]) cudaIpcCloseMemHandle(f->x.peer[p]);
  for (void *p : f->allocs) cudaFree(p);
  delete f;
}

int prism_b200_ffn_exchange_handle(const prism_b200_ffn *f, void *handle) {
  if (!f || !handle) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = f->ex;
  if (f->size < 2) return ex->fail(PRISM_B200_E_INVALID, "FFN chain is not tensor-parallel");
  CK(cudaSetDevice(ex->device), "select device");
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, f->x.base), "exchange handle");
  static_assert(sizeof(h) == PRISM_B200_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return PRISM_B200_OK;
}

int prism_b200_ffn_connect(prism_b200_ffn *f, const void *handles) {
  if (!f || !handles) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = f->ex;
  if (f->size < 2) return ex->fail(PRISM_B200_E_INVALID, "FFN chain is not tensor-parallel");
  if (f->x.connected) return ex->fail(PRISM_B200_E_INVALID, "FFN chain is already connected");
  CK(cudaSetDevice(ex->device), "select device");
  const uint8_t *hb = static_cast<const uint8_t *>(handles);
  for (int p = 0; p < f->size; ++p) {
    if (p == f->rank) {
      f->x.peer[p] = f->x.base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)p * sizeof(h), sizeof(h));
    void *ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return ex->fail(PRISM_B200_E_DEVICE, "open rank %d's exchange buffer: %s", p,
                      cudaGetErrorString(e));
    f->x.peer[p] = static_cast<uint8_t *>(ptr);
    f->x.opened[p] = true;
  }
  f->x.connected = true;
  return PRISM_B200_OK;
}

int prism_b200_ffn_chain_tokens_device(prism_b200_ffn *f, size_t tokens, const float *x_dev,
                                       const float *residual_dev, int pinned, float *out_dev,
                                       void *stream) {
  using namespace prism;
  if (!f) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = f->ex;
  int st = check_open(ex);
  if (st) return st;
  if (tokens == 0) return PRISM_B200_OK;
  if (tokens > f->max_tokens)
    return ex->fail(PRISM_B200_E_INVALID, "at most %zu tokens per call", f->max_tokens);
  if (!x_dev || !out_dev) return ex->fail(PRISM_B200_E_INVALID, "null device buffer");
  if (reinterpret_cast<uintptr_t>(x_dev) % 16 || reinterpret_cast<uintptr_t>(out_dev) % 4 ||
      reinterpret_cast<uintptr_t>(residual_dev) % 4)
    return ex->fail(PRISM_B200_E_INVALID, "misaligned token buffers");
  if (f->size > 1 && !f->x.connected)
    return ex->fail(PRISM_B200_E_INVALID, "connect the ranks before the first call");
  CK(cudaSetDevice(ex->device), "select device");
  cudaStream_t s = pick(ex, stream);
  unsigned *status = ex->d_status;
  const size_t M = tokens;
  const int hnb = f->H / 256, fnb = f->Fl / 256;
  // gate and up over the rank's FFN rows, one quantization of x
  CK(launch_token_quantize(x_dev, M, hnb, pinned, token_q8k_carve(f->tok, M, hnb), status, s,
                           false),
     "quantize");
  const TokenQ8K tx = token_q8k_carve(f->tok, M, hnb);
  CK(launch_token_matmul(f->gate, M, tx, f->g, nullptr, nullptr, status, s, false), "gate");
  CK(launch_token_matmul(f->up, M, tx, f->u, nullptr, nullptr, status, s, false), "up");
  {
    const long n = (long)M * f->Fl;
    swiglu_kernel<<<(unsigned)std::min<long>((n + 255) / 256, 4096), 256, 0, s>>>(f->u, f->g, n,
                                                                                  status);
    CK(cudaGetLastError(), "swiglu");
  }
  CK(launch_token_quantize(f->u, M, fnb, pinned, token_q8k_carve(f->tok, M, fnb), status, s,
                           false),
     "quantize");
  const TokenQ8K th = token_q8k_carve(f->tok, M, fnb);
  if (f->size == 1) {
    CK(launch_token_matmul(f->down, M, th, out_dev, residual_dev, nullptr, status, s, false),
       "down");
  } else {
    // this rank's partial into receive slot `rank` of every rank (slot pair
    // alternating per call), then the rank-ordered sum once all arrived
    const int sl = (int)(f->calls & 1);
    GemmPush push{};
    push.n = f->size;
    push.ld = f->H;
    push.col = 0;
    for (int p = 0; p < f->size; ++p) {
      push.dst[p] = f->x.slot(f->x.peer[p], sl) + (size_t)f->rank * M * f->H;
      push.count[p] = TpExchange::count(f->x.peer[p], 0);
    }
    CK(launch_token_matmul(f->down, M, th, nullptr, nullptr, nullptr, status, s, false, &push),
       "down");
    // the host tracks the counter's target: every rank calls with the same
    // token counts in the same order, as with a collective
    const unsigned long long target = f->delivered + (unsigned long long)f->size * M * f->H;
    const TpWait w{TpExchange::count(f->x.base, 0), f->zero, 0ull, target};
    tp_ffn_reduce_kernel<<<(unsigned)M, 256, 0, s>>>(f->x.slot(f->x.base, sl), f->size, (int)M,
                                                     f->H, w, residual_dev, out_dev, status);
    CK(cudaGetLastError(), "all-reduce");
    f->delivered = target;
  }
  f->calls += 1;
  return PRISM_B200_OK;
}

int prism_b200_ffn_chain_tokens(prism_b200_ffn *f, size_t tokens, const float *x,
                                const float *residual, int pinned, float *out) {
  using namespace prism;
  if (!f) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = f->ex;
  int st = check_open(ex);
  if (st) return st;
  if (tokens == 0) return PRISM_B200_OK;
  if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null token buffer");
  if (tokens > f->max_tokens)
    return ex->fail(PRISM_B200_E_INVALID, "at most %zu tokens per call", f->max_tokens);
  CK(cudaSetDevice(ex->device), "select device");
  const size_t bytes = tokens * f->H * 4;
  CK(ex->tok_x.ensure(2 * bytes), "token input buffer");
  CK(ex->tok_y.ensure(bytes), "token output buffer");
  cudaStream_t s = ex->stream;
  float *xd = static_cast<float *>(ex->tok_x.ptr);
  float *rd = residual ? xd + tokens * f->H : nullptr;
  CK(cudaMemcpyAsync(xd, x, bytes, cudaMemcpyHostToDevice, s), "input copy");
  if (rd) CK(cudaMemcpyAsync(rd, residual, bytes, cudaMemcpyHostToDevice, s), "residual copy");
  if ((st = prism_b200_ffn_chain_tokens_device(f, tokens, xd, rd, pinned,
                                               static_cast<float *>(ex->tok_y.ptr), s)))
    return st;
  CK(cudaMemcpyAsync(out, ex->tok_y.ptr, bytes, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, bytes);
  return st;
}
