// seam.cuh -- the rest of the reference's projection-executor surface.
//
// Included once by prism_b200.cu, after the model and batch code.  These
// entry points complete the mirror of `trait Pq2ProjectionExecutor`
// (reference src/kernels/projection.rs:16-350): the opaque capacity, the
// F32 eligibility queries, sibling projections over token tiles (pair and
// triple), the fused FFN gate/up + SwiGLU for one token and for a token tile,
// and the single-token FFN chain.  Every one validates its arguments before
// any submission, runs the same kernels as the other projections (so every
// output equals, bit for bit, what prism_b200_project_f32_group gives for the
// same token), and closes the executor on a device-side failure.
#pragma once

namespace {

// Geometry of the FFN trio: gate and up [F][H], down [H][F], one kind.
bool ffn_trio_ok(const prism_b200_tensor *gate, const prism_b200_tensor *up,
                 const prism_b200_tensor *down) {
  if (!geometry_ok(gate) || !geometry_ok(up)) return false;
  if (gate->kind != up->kind || gate->rows != up->rows || gate->cols != up->cols) return false;
  if (!down) return true;
  return geometry_ok(down) && down->kind == gate->kind && down->rows == gate->cols &&
         down->cols == gate->rows;
}

prism_b200_tensor tensor_of(const prism_b200_weight *w) {
  prism_b200_tensor t;
  t.kind = w->dw.kind;
  t.cols = w->dw.cols;
  t.rows = w->dw.rows;
  t.data = nullptr;
  return t;
}

// The SwiGLU pair for one token on the device: y = up(x) * silu(gate(x)),
// x quantized to Q8_K in each CTA's prologue (the matvec pair kernel).
cudaError_t swiglu_token_on(prism_b200_executor *ex, const prism_b200_weight *gate,
                            const prism_b200_weight *up, const float *x_dev, int pinned,
                            float *y_dev, cudaStream_t s) {
  MvArgs a;
  a.count = 2;
  a.nb = up->dw.nb;
  a.prologue = kProF32;
  a.in0 = x_dev;
  a.pinned = pinned;
  a.status = ex->d_status;
  a.w[0] = mv_weight(up->dw, y_dev);
  a.w[1] = mv_weight(gate->dw, nullptr);
  return launch_matvec_group(up->dw.kind, kEpiSwiglu, a, ex->num_sms, s, ex->pdl);
}

// Sibling projections over a tile of tokens: the tokens are quantized once,
// then every weight runs on the tensor cores over the same Q8_K tokens.
int project_tokens_group(prism_b200_executor *ex, size_t count,
                         const prism_b200_weight *const *w, size_t tokens, const float *x,
                         int pinned, float *const *outs) {
  int st = check_open(ex);
  if (st) return st;
  if (!w || !outs || count == 0) return ex->fail(PRISM_B200_E_INVALID, "empty group");
  for (size_t i = 0; i < count; ++i) {
    if ((st = validate_weight(ex, w[i]))) return st;
    if (w[i]->dw.cols != w[0]->dw.cols || w[i]->dw.kind != w[0]->dw.kind)
      return ex->fail(PRISM_B200_E_INVALID, "sibling projections must share kind and columns");
    if (!outs[i] && tokens) return ex->fail(PRISM_B200_E_INVALID, "null output");
  }
  if (!tokens) return PRISM_B200_OK;
  if (!x) return ex->fail(PRISM_B200_E_INVALID, "null token buffer");
  if (tokens > (size_t)kMaxTokens)
    return ex->fail(PRISM_B200_E_INVALID, "at most %d tokens per call", kMaxTokens);
  CK(cudaSetDevice(ex->device), "select device");
  const size_t cols = w[0]->dw.cols;
  size_t rows_total = 0;
  for (size_t i = 0; i < count; ++i) rows_total += w[i]->dw.rows;
  const size_t xin = tokens * cols * 4;
  CK(ex->tok_x.ensure(xin), "token input buffer");
  CK(ex->tok_y.ensure(tokens * rows_total * 4), "token output buffer");
  CK(ex->tok_act.ensure(token_q8k_bytes(tokens, (int)(cols / 256))), "token activation buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->tok_x.ptr, x, xin, cudaMemcpyHostToDevice, s), "input copy");
  const TokenQ8K t = token_q8k_carve(ex->tok_act.ptr, tokens, (int)(cols / 256));
  CK(launch_token_quantize(static_cast<const float *>(ex->tok_x.ptr), tokens, (int)(cols / 256),
                           pinned, t, ex->d_status, s, false),
     "token quantize");
  float *y = static_cast<float *>(ex->tok_y.ptr);
  size_t off = 0;
  for (size_t i = 0; i < count; ++i) {
    CK(launch_token_matmul(w[i]->dw, tokens, t, y + off, nullptr, nullptr, ex->d_status, s, false),
       "token projection launch");
    off += tokens * w[i]->dw.rows;
  }
  off = 0;
  for (size_t i = 0; i < count; ++i) {
    const size_t b = tokens * w[i]->dw.rows * 4;
    CK(cudaMemcpyAsync(outs[i], y + off, b, cudaMemcpyDeviceToHost, s), "output copy");
    off += tokens * w[i]->dw.rows;
  }
  st = finish(ex, s);
  if (st)
    for (size_t i = 0; i < count; ++i) memset(outs[i], 0, tokens * w[i]->dw.rows * 4);
  return st;
}

}  // namespace

extern "C" {

int64_t prism_b200_executor_operation_capacity(const prism_b200_executor *ex) {
  // resident weights and device-side work queues: no bounded session
  (void)ex;
  return -1;
}

int prism_b200_executor_supports_f32(const prism_b200_executor *ex,
                                     const prism_b200_tensor *tensor) {
  return prism_b200_executor_supports(ex, tensor);
}

int prism_b200_executor_supports_f32_group(const prism_b200_executor *ex, size_t count,
                                           const prism_b200_tensor *const *tensors) {
  if (!ex || !tensors || count == 0 || count > 4) return 0;
  for (size_t i = 0; i < count; ++i)
    if (!geometry_ok(tensors[i]) || tensors[i]->kind != tensors[0]->kind ||
        tensors[i]->cols != tensors[0]->cols)
      return 0;
  return 1;
}

int prism_b200_executor_supports_q8(const prism_b200_executor *ex,
                                    const prism_b200_tensor *tensor) {
  // Q8_0 activations serve PTQ1 and PQ2 rows (the reference routes PQ2 here
  // when its columns are not a multiple of 256); TQ2_0, TQ1_0 and the K
  // quants take Q8_K
  return ex && pq_geometry_ok(tensor) ? 1 : 0;
}

int prism_b200_project_q8(prism_b200_executor *ex, const prism_b200_weight *w,
                          const void *activation, int pinned, float *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_any_weight(ex, w))) return st;
  const DeviceWeight &dw = w->dw;
  const size_t ybytes = dw.rows * sizeof(float);
  if (!dw.packed || kquant_block_bytes(dw.kind)) {
    if (out) memset(out, 0, ybytes);
    return ex->fail(PRISM_B200_E_UNSUPPORTED,
                    "kind %u takes Q8_K activations (prism_b200_project), not Q8_0", dw.kind);
  }
  if (pinned) {
    if (out) memset(out, 0, ybytes);
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "pinned accumulation of kind %u", dw.kind);
  }
  if (!activation || !out) return ex->fail(PRISM_B200_E_INVALID, "null buffer");
  const size_t abytes = dw.cols / 32 * sizeof(Q8Act);
  CK(cudaSetDevice(ex->device), "select device");
  CK(ex->act.ensure(abytes), "activation buffer");
  CK(ex->y.ensure(ybytes), "output buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->act.ptr, activation, abytes, cudaMemcpyHostToDevice, s),
     "activation copy");
  CK(launch_packed(ex, dw, ex->act.ptr, false, 0, static_cast<float *>(ex->y.ptr), s),
     "packed matvec launch");
  CK(cudaMemcpyAsync(out, ex->y.ptr, ybytes, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, ybytes);
  return st;
}

int prism_b200_executor_supports_tile_tokens(const prism_b200_executor *ex) { return ex ? 1 : 0; }

int prism_b200_project_f32_pair_tokens(prism_b200_executor *ex,
                                       const prism_b200_weight *const *weights, size_t tokens,
                                       const float *x, int pinned, float *out_a, float *out_b) {
  float *outs[2] = {out_a, out_b};
  return project_tokens_group(ex, 2, weights, tokens, x, pinned, outs);
}

int prism_b200_project_f32_triple_tokens(prism_b200_executor *ex,
                                         const prism_b200_weight *const *weights, size_t tokens,
                                         const float *x, int pinned, float *out_a, float *out_b,
                                         float *out_c) {
  float *outs[3] = {out_a, out_b, out_c};
  return project_tokens_group(ex, 3, weights, tokens, x, pinned, outs);
}

int prism_b200_executor_supports_f32_ffn_swiglu(const prism_b200_executor *ex,
                                                const prism_b200_tensor *gate,
                                                const prism_b200_tensor *up) {
  return ex && ffn_trio_ok(gate, up, nullptr) ? 1 : 0;
}

int prism_b200_project_f32_ffn_swiglu(prism_b200_executor *ex, const prism_b200_weight *gate,
                                      const prism_b200_weight *up, const float *x, int pinned,
                                      float *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, gate)) || (st = validate_weight(ex, up))) return st;
  const prism_b200_tensor tg = tensor_of(gate), tu = tensor_of(up);
  if (!ffn_trio_ok(&tg, &tu, nullptr) || gate->dw.h != up->dw.h)
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "gate and up must share kind and geometry");
  if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null buffer");
  CK(cudaSetDevice(ex->device), "select device");
  const size_t n = up->dw.cols, rows = up->dw.rows;
  CK(ex->x.ensure(n * 4), "input buffer");
  CK(ex->y.ensure(rows * 4), "output buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->x.ptr, x, n * 4, cudaMemcpyHostToDevice, s), "input copy");
  CK(swiglu_token_on(ex, gate, up, static_cast<const float *>(ex->x.ptr), pinned,
                     static_cast<float *>(ex->y.ptr), s),
     "SwiGLU pair launch");
  CK(cudaMemcpyAsync(out, ex->y.ptr, rows * 4, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, rows * 4);
  return st;
}

int prism_b200_project_f32_ffn_swiglu_tokens(prism_b200_executor *ex,
                                             const prism_b200_weight *gate,
                                             const prism_b200_weight *up, size_t tokens,
                                             const float *x, int pinned, float *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, gate)) || (st = validate_weight(ex, up))) return st;
  const prism_b200_tensor tg = tensor_of(gate), tu = tensor_of(up);
  if (!ffn_trio_ok(&tg, &tu, nullptr))
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "gate and up must share kind and geometry");
  if (!tokens) return PRISM_B200_OK;
  if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null token buffer");
  if (tokens > (size_t)kMaxTokens)
    return ex->fail(PRISM_B200_E_INVALID, "at most %d tokens per call", kMaxTokens);
  CK(cudaSetDevice(ex->device), "select device");
  const size_t cols = up->dw.cols, rows = up->dw.rows, nb = cols / 256;
  const size_t xin = tokens * cols * 4, yout = tokens * rows * 4;
  CK(ex->tok_x.ensure(xin), "token input buffer");
  CK(ex->tok_y.ensure(2 * yout), "token output buffer");
  CK(ex->tok_act.ensure(token_q8k_bytes(tokens, (int)nb)), "token activation buffer");
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(ex->tok_x.ptr, x, xin, cudaMemcpyHostToDevice, s), "input copy");
  const TokenQ8K t = token_q8k_carve(ex->tok_act.ptr, tokens, (int)nb);
  CK(launch_token_quantize(static_cast<const float *>(ex->tok_x.ptr), tokens, (int)nb, pinned, t,
                           ex->d_status, s, false),
     "token quantize");
  float *u = static_cast<float *>(ex->tok_y.ptr), *g = u + tokens * rows;
  CK(launch_token_matmul(up->dw, tokens, t, u, nullptr, nullptr, ex->d_status, s, false),
     "up projection");
  CK(launch_token_matmul(gate->dw, tokens, t, g, nullptr, nullptr, ex->d_status, s, false),
     "gate projection");
  const long n = (long)(tokens * rows);
  swiglu_kernel<<<(unsigned)std::min<long>((n + 255) / 256, 4096), 256, 0, s>>>(u, g, n,
                                                                                ex->d_status);
  CK(cudaGetLastError(), "SwiGLU");
  CK(cudaMemcpyAsync(out, u, yout, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, yout);
  return st;
}

int prism_b200_executor_supports_f32_ffn_chain(const prism_b200_executor *ex,
                                               const prism_b200_tensor *gate,
                                               const prism_b200_tensor *up,
                                               const prism_b200_tensor *down) {
  return ex && down && ffn_trio_ok(gate, up, down) ? 1 : 0;
}

int prism_b200_project_f32_ffn_chain(prism_b200_executor *ex, const prism_b200_weight *gate,
                                     const prism_b200_weight *up, const prism_b200_weight *down,
                                     const float *x, const float *residual,
                                     uint32_t hadamard_block_size, int pinned, float *out) {
  int st = check_open(ex);
  if (st) return st;
  if ((st = validate_weight(ex, gate)) || (st = validate_weight(ex, up)) ||
      (st = validate_weight(ex, down)))
    return st;
  const prism_b200_tensor tg = tensor_of(gate), tu = tensor_of(up), td = tensor_of(down);
  if (!ffn_trio_ok(&tg, &tu, &td) || gate->dw.h != up->dw.h)
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "gate/up [F][H] and down [H][F] of one kind");
  if (hadamard_block_size)
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "Hadamard-rotated FFN chains are not served");
  if (!x || !out) return ex->fail(PRISM_B200_E_INVALID, "null buffer");
  CK(cudaSetDevice(ex->device), "select device");
  const size_t H = up->dw.cols, F = up->dw.rows;
  CK(ex->x.ensure((2 * H + F) * 4), "input buffer");
  CK(ex->y.ensure(H * 4), "output buffer");
  float *xd = static_cast<float *>(ex->x.ptr), *rd = xd + H, *hd = xd + 2 * H;
  cudaStream_t s = ex->stream;
  CK(cudaMemcpyAsync(xd, x, H * 4, cudaMemcpyHostToDevice, s), "input copy");
  if (residual) CK(cudaMemcpyAsync(rd, residual, H * 4, cudaMemcpyHostToDevice, s), "residual copy");
  CK(swiglu_token_on(ex, gate, up, xd, pinned, hd, s), "SwiGLU pair launch");
  MvArgs a;
  a.count = 1;
  a.nb = down->dw.nb;
  a.prologue = kProF32;
  a.in0 = hd;
  a.pinned = pinned;
  a.status = ex->d_status;
  a.w[0] = mv_weight(down->dw, static_cast<float *>(ex->y.ptr), residual ? rd : nullptr);
  CK(launch_matvec_group(down->dw.kind, kEpiStore, a, ex->num_sms, s, ex->pdl), "down launch");
  CK(cudaMemcpyAsync(out, ex->y.ptr, H * 4, cudaMemcpyDeviceToHost, s), "output copy");
  st = finish(ex, s);
  if (st) memset(out, 0, H * 4);
  return st;
}

}  // extern "C"

// ---- measured dense int8 tensor-core rate ----------------------------------
// No reference counterpart: the denominator of the GEMM's tensor roofline.
// One CTA per SM issues `iters` back-to-back kind::i8 MMAs (128x256x32) from
// shared memory; a warm-up launch precedes the event-timed one.
extern "C" int prism_b200_tensor_peak_i8(prism_b200_executor *ex, int iters, double *tops) {
  int st = check_open(ex);
  if (st) return st;
  if (!tops || iters < 1 || iters > (1 << 20))
    return ex->fail(PRISM_B200_E_INVALID, "iters must be 1..2^20 and tops non-null");
  CK(cudaSetDevice(ex->device), "select device");
  cudaStream_t s = ex->stream;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  CK(cudaEventCreate(&e0), "event");
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return ex->fail(PRISM_B200_E_DEVICE, "event");
  }
  tensor_peak_i8_kernel<<<ex->num_sms, 128, 0, s>>>(iters, ex->d_status);
  cudaEventRecord(e0, s);
  tensor_peak_i8_kernel<<<ex->num_sms, 128, 0, s>>>(iters, ex->d_status);
  cudaEventRecord(e1, s);
  cudaError_t e = cudaGetLastError();
  st = e == cudaSuccess ? finish(ex, s) : cuda_fail(ex, e, "tensor peak launch");
  float ms = 0.0f;
  if (st == PRISM_B200_OK && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess && ms > 0.0f)
    *tops = 2.0 * kPeakM * kPeakN * kPeakK * (double)iters * ex->num_sms / (ms * 1e-3) / 1e12;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return st;
}
