// batch.cuh -- batched serving: many sequences decoded together over one
// model's resident weights.
//
// Every step advances each of B sequences by one token.  The projections of
// all B tokens run as tensor-core GEMMs (gemm.cuh: 128 tokens x 128 rows
// per CTA, tcgen05.mma kind::i8), so a weight byte is read once per step for
// the whole batch instead of once per sequence; Gated DeltaNet and attention
// run per (sequence, head) on each sequence's own state and KV cache.
// Each sequence's results are those of decoding it alone -- the reference's
// weight-sharing batched evaluation contract (reference src/lib.rs:255-275
// `evaluate_batch_into`: "final decoder state matches sequential
// evaluation"); the server keeps one decoder per sequence
// (reference server/src/native_backend).  Included once by prism_b200.cu,
// after model.cuh.
#pragma once

#include "gemm.cuh"
#include "serve_attn.cuh"
#include "tp.cuh"

namespace prism {

struct BatchLayer {
  float *conv = nullptr;                  // 2 x [B][channels][k-1], by step parity
  float *matrix = nullptr;                // [B][values][S][S]
  // binary16: [B][context][kv heads * hd]; Q8_0 with the serving kernel:
  // [B][kv head][context][record]
  uint16_t *kc = nullptr, *vc = nullptr;
};

// The weights one rank multiplies by: the model's own (one rank) or its
// tensor-parallel slices (tp.cuh), with the per-head vectors of its heads.
struct ShardLayer {
  DeviceWeight q, k, v, o, qkv, z, beta, alpha, out, up, gate, down;
  const float *conv_w = nullptr, *dt_bias = nullptr, *ssm_a = nullptr;
};

}  // namespace prism

struct prism_b200_batch {
  prism_b200_model *m = nullptr;
  int B = 0, context = 0;
  std::vector<prism::BatchLayer> L;
  // activations [B][...]
  float *hidden = nullptr, *xn = nullptr, *mixed = nullptr, *zgate = nullptr, *beta = nullptr,
        *alpha = nullptr, *attended = nullptr, *projected = nullptr, *key = nullptr,
        *value = nullptr, *up = nullptr, *gate = nullptr;
  void *tok = nullptr;  // Q8_K tokens for the GEMMs (largest K)
  int *d_pos = nullptr, *d_step = nullptr;
  uint32_t *d_tokens = nullptr;
  unsigned long long *d_keys = nullptr;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t graph = nullptr;
  std::vector<void *> allocations;
  int64_t steps = 0;
  bool serve_attn = false;  // Q8_0 KV through attention_serve_kernel (head-major cache)
  // tensor parallelism: this rank's slice; one rank owns everything
  prism::TpPlan tp;
  std::vector<prism::ShardLayer> S;
  prism::DeviceWeight lm;   // output head rows [tp.v0, tp.v1)
  prism::TpExchange x;
  int heads = 0, kv_heads = 0, gdn_groups = 0, gdn_heads = 0, ffn = 0;  // this rank's
  size_t kv_row = 0;        // bytes of one cached position of this rank's KV heads
  size_t kv_seq_bytes() const { return (size_t)context * kv_row; }
  int gdn_width() const { return gdn_heads * (int)m->cfg.ssm_state; }
  int gdn_channels() const { return (2 * gdn_groups + gdn_heads) * (int)m->cfg.ssm_state; }
};

namespace prism {

template <typename T>
cudaError_t batch_alloc(prism_b200_batch *b, T **p, size_t count) {
  void *v = nullptr;
  const size_t bytes = count * sizeof(T) < 16 ? 16 : count * sizeof(T);
  cudaError_t e = cudaMalloc(&v, bytes);
  if (e != cudaSuccess) return e;
  b->allocations.push_back(v);
  e = cudaMemset(v, 0, bytes);
  *p = static_cast<T *>(v);
  return e;
}

template <int KIND>
__global__ void embed_batch_kernel(const uint8_t *units, int h, int nb, int vocab,
                                   const uint32_t *tokens, float *hidden, int n,
                                   unsigned *status) {
  grid_dependency_wait();
  grid_dependents_launch();
  const int b = blockIdx.y;
  const uint32_t token = tokens[b];
  if (token >= (uint32_t)vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(status, kStatusInvalid);
    return;
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    hidden[(long)b * n + i] = decode_tiled<KIND>(units, h, nb, (int)token, i);
}

// RMSNorm of each row (one 256-thread CTA per row): the binary64 sum of
// squares in block_sumsq_f64's order, then (x * scale) * w -- the values the
// projection kernels' RMSNorm prologue quantizes.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float *x, const float *w, int n,
                                                           float eps, float *out,
                                                           unsigned *status) {
  __shared__ double red[8];
  grid_dependency_wait();
  grid_dependents_launch();
  const float *xr = x + (long)blockIdx.x * n;
  const double sum = block_sumsq_f64(xr, n, red);
  const float mean = (float)(sum / (double)n);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  if ((!is_finite_f(scale) || !(scale > 0.0f)) && threadIdx.x == 0) report(status, kStatusNonfinite);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[(long)blockIdx.x * n + i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

// h = up * silu(gate) (reference src/graph.rs:121-131 SwiGLU), in place over up.
__global__ void swiglu_kernel(float *up, const float *gate, long n, unsigned *status) {
  grid_dependency_wait();
  grid_dependents_launch();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const float u = up[i], g = gate[i];
    if (!is_finite_f(u) || !is_finite_f(g)) report(status, kStatusNonfinite);
    up[i] = __fmul_rn(u, silu_f(g));
  }
}

// Advance every sequence; with `greedy`, its next input is the argmax token.
__global__ void batch_finish_kernel(unsigned long long *keys, uint32_t *tokens, int *pos, int B,
                                    int *step, int greedy) {
  grid_dependency_wait();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    if (greedy) tokens[b] = 0xffffffffu - (unsigned)(keys[b] & 0xffffffffull);
    keys[b] = 0ull;
    pos[b] += 1;
  }
  if (threadIdx.x == 0) *step += 1;
}

// Seeded synthetic context for benchmarks: every sequence at `position`
// with random KV rows (binary16 in [-1, 1], or Q8_0 records with scales in
// [2^-8, 2^-6] and codes in [-127, 127]) and small random recurrent and
// convolution states.  SplitMix64 of (seed, array, element).
__device__ __forceinline__ uint64_t synth_mix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

// q8: 1 plain Q8_0 records, 2 K pages of kServePage interleaved records
__global__ void fill_kv_kernel(uint8_t *kv, long rows, int row_bytes, int hd, int q8,
                               uint64_t seed) {
  const long n = rows * row_bytes;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const uint64_t r = synth_mix(seed ^ (uint64_t)i);
    uint8_t v;
    if (q8) {
      const int rb = q8_0_record_bytes(hd);
      const bool scale_byte = q8 == 2 ? (int)(i % ((long)kServePage * rb)) < kServePage * (hd / 32) * 2
                                      : (int)((i % row_bytes) % rb) < hd / 32 * 2;
      const int o = (int)(i & 1);
      if (scale_byte) {
        // binary16 scale in [2^-8, 2^-6): exponent 7..8, random mantissa
        const uint16_t half = (uint16_t)((7u + (unsigned)(r & 1)) << 10 | (unsigned)((r >> 8) & 0x3ff));
        v = (o & 1) ? (uint8_t)(half >> 8) : (uint8_t)(half & 0xff);
      } else {
        v = (uint8_t)(int8_t)((int)(r % 255) - 127);
      }
    } else {
      // binary16 in (-1, 1): sign, exponent < 15, random mantissa
      const uint16_t half = (uint16_t)(((r >> 20) & 1) << 15 | ((r % 15) << 10) | ((r >> 8) & 0x3ff));
      v = (i & 1) ? (uint8_t)(half >> 8) : (uint8_t)(half & 0xff);
    }
    kv[i] = v;
  }
}

__global__ void fill_f32_kernel(float *x, long n, float scale, uint64_t seed) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    const uint64_t r = synth_mix(seed ^ (uint64_t)i);
    x[i] = scale * ((float)(r >> 40) * (1.0f / 16777216.0f) * 2.0f - 1.0f);
  }
}

// Enqueue one step of the whole batch on b->stream.
inline cudaError_t enqueue_batch_step(prism_b200_batch *b, bool greedy) {
  prism_b200_model *m = b->m;
  prism_b200_executor *ex = m->ex;
  const auto &c = m->cfg;
  const bool pdl = ex->pdl;
  const int B = b->B;
  cudaStream_t s = b->stream;
  unsigned *status = ex->d_status;
  const uint32_t kind = c.weight_kind;
  cudaLaunchAttribute attr[2];
  cudaError_t e;
  const int H = (int)c.hidden, hnb = H / 256;
  {
    cudaLaunchConfig_t cfg = pdl_config(dim3((H + 255) / 256, B), dim3(256), 0, s, attr, pdl);
    e = kind == 35 ? cudaLaunchKernelEx(&cfg, embed_batch_kernel<35>, m->embd.units, m->embd.h,
                                        m->embd.nb, (int)c.vocab, (const uint32_t *)b->d_tokens,
                                        b->hidden, H, status)
                   : cudaLaunchKernelEx(&cfg, embed_batch_kernel<10>, m->embd.units, m->embd.h,
                                        m->embd.nb, (int)c.vocab, (const uint32_t *)b->d_tokens,
                                        b->hidden, H, status);
    if (e != cudaSuccess) return e;
  }
  const bool tpx = b->tp.size > 1;
  const bool exact = tpx && b->x.mode == kTpExact;
  const int ranks = b->tp.size;
  const int hd = (int)c.head_dim;
  const unsigned long long MH = (unsigned long long)B * H;
  // Exchanges of this step (tensor parallelism): values delivered to each
  // counter per step and so far in this step.  A projection that leaves the
  // heads or the FFN marks its exchange pending; the next normalisation
  // waits for it (and, all-reduce, sums the partials).
  unsigned long long gather_step = 0, gather_done = 0, hidden_done = 0;
  for (size_t l = 0; l < m->L.size(); ++l)
    gather_step += (unsigned long long)B *
                   ((m->L[l].full ? c.heads * c.head_dim : (uint32_t)m->value_width()) / 256 +
                    c.ffn / 256);
  int pending = -1, pending_index = 0;
  auto norm = [&](const float *w) {
    if (pending < 0) {
      cudaLaunchConfig_t cfg = pdl_config(dim3(B), dim3(256), 0, s, attr, pdl);
      return cudaLaunchKernelEx(&cfg, rmsnorm_rows_kernel, (const float *)b->hidden, w, H, c.eps,
                                b->xn, status);
    }
    TpWait tw;
    const float *slot = nullptr;
    int nr = 0;
    if (exact) {
      tw = TpWait{TpExchange::count(b->x.base, 0), b->x.xstep, 2ull * c.layers * MH, hidden_done};
    } else {
      tw = TpWait{TpExchange::count(b->x.base, pending), b->x.xstep,
                  (unsigned long long)c.layers * ranks * MH,
                  (unsigned long long)(pending_index + 1) * ranks * MH};
      slot = b->x.slot(b->x.base, pending);
      nr = ranks;
    }
    pending = -1;
    cudaLaunchConfig_t cfg = pdl_config(dim3(B), dim3(256), 0, s, attr, pdl);
    return cudaLaunchKernelEx(&cfg, tp_reduce_norm_kernel, slot, nr, B, H, tw, b->hidden, w,
                              c.eps, b->xn, status);
  };
  auto quant = [&](const float *x, int nb) {
    return launch_token_quantize(x, B, nb, 0, token_q8k_carve(b->tok, B, nb), status, s, pdl);
  };
  auto mm = [&](const DeviceWeight &w, float *y, const float *residual,
                unsigned long long *keys, int row_base = 0) {
    return launch_token_matmul(w, B, token_q8k_carve(b->tok, B, w.nb), y, residual, keys,
                               status, s, pdl, nullptr, row_base);
  };
  // hidden += Q8_K(x) W^T for the projections leaving the heads / the FFN.
  // x is this rank's [B][nbl * 256] part, blocks b0.. of the full nbt.
  auto project_out = [&](const DeviceWeight &w, const float *x, int nbl, int b0, int nbt,
                         int slot, int index) -> cudaError_t {
    cudaError_t e2;
    if (!tpx) {
      if ((e2 = quant(x, nbl)) != cudaSuccess) return e2;
      return mm(w, b->hidden, b->hidden, nullptr);
    }
    if (!exact) {
      // row-parallel partial into every rank's slot
      if ((e2 = quant(x, nbl)) != cudaSuccess) return e2;
      const GemmPush push = b->x.push_partial(b->tp.rank, slot);
      pending = slot;
      pending_index = index;
      return launch_token_matmul(w, B, token_q8k_carve(b->tok, B, w.nb), nullptr, nullptr,
                                 nullptr, status, s, pdl, &push, 0);
    }
    // exact: gather every rank's quantized blocks, then this rank's hidden
    // rows (with the residual) into every rank's hidden state
    TpGather gq{};
    gq.ranks = ranks;
    for (int p = 0; p < ranks; ++p) {
      gq.dst[p] = token_q8k_carve(b->x.tok(b->x.peer[p]), B, nbt);
      gq.count[p] = TpExchange::count(b->x.peer[p], 3);
    }
    {
      const long warps = (long)B * nbl;
      cudaLaunchConfig_t cfg =
          pdl_config(dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, s, attr, pdl);
      if ((e2 = cudaLaunchKernelEx(&cfg, q8k_gather_kernel, x, B, nbl, b0, nbt, gq, status)) !=
          cudaSuccess)
        return e2;
    }
    gather_done += (unsigned long long)B * nbt;
    const TpWait gate{TpExchange::count(b->x.base, 3), b->x.xstep, gather_step, gather_done};
    const GemmPush push = b->x.push_rows(b->tp.hr0);
    hidden_done += MH;
    pending = 0;
    return launch_token_matmul(w, B, token_q8k_carve(b->x.tok(b->x.base), B, nbt), nullptr,
                               b->hidden, nullptr, status, s, pdl, &push, 0, &gate);
  };
#define BK(x)                            \
  if ((e = (x)) != cudaSuccess) return e
  for (size_t l = 0; l < m->L.size(); ++l) {
    ModelLayer &Ly = m->L[l];
    ShardLayer &Sh = b->S[l];
    BatchLayer &Bl = b->L[l];
    BK(norm(Ly.attn_norm));
    BK(quant(b->xn, hnb));
    if (Ly.full) {
      BK(mm(Sh.q, b->projected, nullptr, nullptr));
      BK(mm(Sh.k, b->key, nullptr, nullptr));
      BK(mm(Sh.v, b->value, nullptr, nullptr));
      AttnArgs aa{};
      aa.heads = b->heads;
      aa.kv_heads = b->kv_heads;
      aa.hd = (int)c.head_dim;
      aa.rope_dim = (int)c.rope_dim;
      for (int j = 0; j < 3; ++j) aa.sections[j] = (int)c.rope_sections[j];
      aa.eps = c.eps;
      aa.theta_scale = powf(c.rope_base, -2.0f / (float)c.rope_dim);
      aa.projected = b->projected;
      aa.key_in = b->key;
      aa.value_in = b->value;
      aa.q_norm = Ly.q_norm;
      aa.k_norm = Ly.k_norm;
      aa.kcache = Bl.kc;
      aa.vcache = Bl.vc;
      aa.q8 = c.kv_policy == PRISM_B200_KV_Q8_0 ? 1 : 0;
      aa.position = b->d_pos;
      aa.pos_stride = 1;
      aa.seq_proj = (long)b->heads * c.head_dim * 2;
      aa.seq_kv_in = (long)b->kv_heads * c.head_dim;
      aa.seq_out = (long)b->heads * c.head_dim;
      aa.seq_cache = (long)(b->kv_seq_bytes() / 2);
      aa.attended = b->attended;
      aa.status = status;
      if (b->serve_attn) {
        // one cluster per (sequence, KV head) over the head-major cache
        ServeArgs sa{aa, b->context};
        const size_t smem = serve_smem_bytes((int)c.head_dim, b->context);
        cudaLaunchConfig_t cfg = pdl_config(dim3(kServeSplit, b->kv_heads, B),
                                            dim3(kServeThreads), smem, s, attr, pdl);
        attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = kServeSplit;
        attr[cfg.numAttrs].val.clusterDim.y = 1;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs += 1;
        BK(cudaLaunchKernelEx(&cfg, attention_serve_kernel, sa));
      } else {
        const size_t smem = attn_launch_smem(aa, b->context);
        cudaLaunchConfig_t cfg =
            pdl_config(dim3(b->heads * kAttnSplit, B), dim3(kAttnThreads), smem, s, attr, pdl);
        attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = kAttnSplit;
        attr[cfg.numAttrs].val.clusterDim.y = 1;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs += 1;
        BK(cudaLaunchKernelEx(&cfg, attention_decode_kernel, aa));
      }
      BK(project_out(Sh.o, b->attended, b->heads * hd / 256, b->tp.qh0 * hd / 256,
                     (int)(c.heads * c.head_dim / 256), 0, (int)l));
    } else {
      BK(mm(Sh.qkv, b->mixed, nullptr, nullptr));
      BK(mm(Sh.z, b->zgate, nullptr, nullptr));
      BK(mm(Sh.beta, b->beta, nullptr, nullptr));
      BK(mm(Sh.alpha, b->alpha, nullptr, nullptr));
      GdnArgs g{};
      g.S = (int)c.ssm_state;
      g.groups = b->gdn_groups;
      g.values = b->gdn_heads;
      g.conv_k = (int)c.conv_kernel;
      g.eps = c.eps;
      g.mixed = b->mixed;
      g.zgate = b->zgate;
      g.beta_in = b->beta;
      g.alpha_in = b->alpha;
      g.in_stride = b->gdn_channels();
      g.z_stride = b->gdn_width();
      g.ab_stride = b->gdn_heads;
      g.conv_w = Sh.conv_w;
      g.dt_bias = Sh.dt_bias;
      g.ssm_a = Sh.ssm_a;
      g.norm_w = Ly.ssm_norm;
      g.conv_state = Bl.conv;
      g.conv_stride = (long)b->gdn_channels() * (c.conv_kernel - 1);
      g.conv_buf_stride = g.conv_stride * B;
      g.state = Bl.matrix;
      g.state_stride = (long)b->gdn_heads * c.ssm_state * c.ssm_state;
      g.attended = b->attended;
      g.out_stride = b->gdn_width();
      g.position = b->d_step;  // the double-buffered history alternates every step
      g.status = status;
      cudaLaunchConfig_t cfg =
          pdl_config(dim3(b->gdn_heads, B), dim3(kGdnThreads), 0, s, attr, pdl);
      BK(cudaLaunchKernelEx(&cfg, gdn_decode_kernel, g));
      BK(project_out(Sh.out, b->attended, b->gdn_width() / 256,
                     b->tp.gh0 * (int)c.ssm_state / 256, m->value_width() / 256, 0, (int)l));
    }
    BK(norm(Ly.post_norm));
    BK(quant(b->xn, hnb));
    BK(mm(Sh.up, b->up, nullptr, nullptr));
    BK(mm(Sh.gate, b->gate, nullptr, nullptr));
    {
      const long n = (long)B * b->ffn;
      cudaLaunchConfig_t cfg =
          pdl_config(dim3((unsigned)std::min<long>((n + 255) / 256, 4096)), dim3(256), 0, s,
                     attr, pdl);
      BK(cudaLaunchKernelEx(&cfg, swiglu_kernel, b->up, (const float *)b->gate, n, status));
    }
    BK(project_out(Sh.down, b->up, b->ffn / 256, b->tp.fb0, (int)(c.ffn / 256), 1, (int)l));
  }
  if (greedy) {
    BK(norm(m->out_norm));
    BK(quant(b->xn, hnb));
    BK(mm(b->lm, nullptr, nullptr, b->d_keys, b->tp.v0));
  } else if (pending >= 0) {
    BK(norm(nullptr));  // the last exchange still has to reach the hidden state
  }
  cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(256), 0, s, attr, pdl);
  if (tpx) {
    TpKeys kp{};
    for (int p = 0; p < b->tp.size; ++p) {
      kp.dst[p] = b->x.keys(b->x.peer[p]) + (size_t)b->tp.rank * B;
      kp.count[p] = TpExchange::count(b->x.peer[p], 2);
    }
    // every rank adds 1 per step
    const TpWait kw{TpExchange::count(b->x.base, 2), b->x.xstep, (unsigned long long)ranks,
                    (unsigned long long)ranks};
    BK(cudaLaunchKernelEx(&cfg, tp_finish_kernel, b->d_keys, kp,
                          (const unsigned long long *)b->x.keys(b->x.base), b->tp.size, kw,
                          b->d_tokens, b->d_pos, B, b->d_step, b->x.xstep, greedy ? 1 : 0,
                          status));
  } else {
    BK(cudaLaunchKernelEx(&cfg, batch_finish_kernel, b->d_keys, b->d_tokens, b->d_pos, B,
                          b->d_step, greedy ? 1 : 0));
  }
#undef BK
  return cudaSuccess;
}

}  // namespace prism

extern "C" {

int prism_b200_batch_create(prism_b200_model *m, uint32_t sequences, uint32_t context,
                            prism_b200_batch **out) {
  return prism_b200_batch_create_tp(m, sequences, context, 0, 1, PRISM_B200_TP_EXACT, out);
}

int prism_b200_batch_create_tp(prism_b200_model *m, uint32_t sequences, uint32_t context,
                               uint32_t tp_rank, uint32_t tp_size, uint32_t tp_mode,
                               prism_b200_batch **out) {
  using namespace prism;
  if (!m || !out) return PRISM_B200_E_INVALID;
  *out = nullptr;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (sequences == 0 || sequences > 65535u || context == 0 ||
      context > (1u << 20))
    return ex->fail(PRISM_B200_E_INVALID, "batch of %u sequences x %u positions", sequences,
                    context);
  if ((context + kAttnSplit - 1) / kAttnSplit + 1 > 16384)
    return ex->fail(PRISM_B200_E_UNSUPPORTED, "context %u exceeds the attention kernel", context);
  const auto &c = m->cfg;
  if (m->rotated())
    return ex->fail(PRISM_B200_E_UNSUPPORTED,
                    "batched serving keeps binary16 or Q8_0 KV, not rotated records");
  if (tp_mode != PRISM_B200_TP_EXACT && tp_mode != PRISM_B200_TP_ALLREDUCE)
    return ex->fail(PRISM_B200_E_INVALID, "tensor-parallel mode %u", tp_mode);
  const bool allreduce = tp_mode == PRISM_B200_TP_ALLREDUCE;
  TpPlan plan;
  if (const char *why = tp_plan(c, (int)tp_rank, (int)tp_size, plan))
    return ex->fail(tp_size < 1 || tp_size > (uint32_t)kMaxTp || tp_rank >= tp_size
                        ? PRISM_B200_E_INVALID
                        : PRISM_B200_E_UNSUPPORTED,
                    "tensor parallelism %u/%u: %s", tp_rank, tp_size, why);
  cudaSetDevice(ex->device);
  auto *b = new prism_b200_batch();
  b->m = m;
  b->B = (int)sequences;
  b->context = (int)context;
  b->tp = plan;
  const bool tpx = plan.size > 1;
  b->heads = plan.qh1 - plan.qh0;
  b->kv_heads = plan.kv1 - plan.kv0;
  b->gdn_heads = tpx ? plan.gh1 - plan.gh0 : (int)c.ssm_values;
  b->gdn_groups = tpx ? b->gdn_heads : (int)c.ssm_groups;
  b->ffn = (plan.fb1 - plan.fb0) * 256;
  b->kv_row = m->kv_row_bytes() / c.kv_heads * b->kv_heads;
  b->serve_attn = c.kv_policy == PRISM_B200_KV_Q8_0 && b->heads / b->kv_heads <= kServeGroup &&
                  context % kServeChunk == 0 &&
                  c.head_dim == (uint32_t)kServeThreads &&
                  serve_smem_bytes((int)c.head_dim, (int)context) <= (size_t)kMaxSmem;
  if (b->serve_attn &&
      cudaFuncSetAttribute(attention_serve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)serve_smem_bytes((int)c.head_dim, (int)context)) != cudaSuccess)
    b->serve_attn = false;
  b->L.resize(c.layers);
  const size_t B = sequences;
  cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
  // this rank's weights: the model's own, or gathered slices
  b->S.resize(c.layers);
  const int S = (int)c.ssm_state, hd = (int)c.head_dim;
  for (uint32_t l = 0; l < c.layers && e == cudaSuccess; ++l) {
    const ModelLayer &Ly = m->L[l];
    ShardLayer &Sh = b->S[l];
    if (!tpx) {
      Sh.q = Ly.q; Sh.k = Ly.k; Sh.v = Ly.v; Sh.o = Ly.o;
      Sh.qkv = Ly.qkv; Sh.z = Ly.z; Sh.beta = Ly.beta; Sh.alpha = Ly.alpha; Sh.out = Ly.out;
      Sh.up = Ly.up; Sh.gate = Ly.gate; Sh.down = Ly.down;
      Sh.conv_w = Ly.conv_w; Sh.dt_bias = Ly.dt_bias; Sh.ssm_a = Ly.ssm_a;
      continue;
    }
    auto gather = [&](const DeviceWeight &w, const std::vector<int> &rows, int b0, int nb,
                      DeviceWeight &o) {
      if (e == cudaSuccess)
        e = tp_gather_weight(w, rows, b0, nb, ex->num_sms, b->allocations, b->stream, o);
    };
    if (Ly.full) {
      // q rows interleave [query(hd) | gate(hd)] per head
      gather(Ly.q, tp_rows({{plan.qh0 * 2 * hd, plan.qh1 * 2 * hd}}), 0, Ly.q.nb, Sh.q);
      gather(Ly.k, tp_rows({{plan.kv0 * hd, plan.kv1 * hd}}), 0, Ly.k.nb, Sh.k);
      gather(Ly.v, tp_rows({{plan.kv0 * hd, plan.kv1 * hd}}), 0, Ly.v.nb, Sh.v);
      if (allreduce)  // input blocks of this rank's heads
        gather(Ly.o, tp_rows({{0, (int)c.hidden}}), plan.qh0 * hd / 256,
               (plan.qh1 - plan.qh0) * hd / 256, Sh.o);
      else  // this rank's hidden rows over every input block
        gather(Ly.o, tp_rows({{plan.hr0, plan.hr1}}), 0, Ly.o.nb, Sh.o);
    } else {
      const int kw = (int)c.ssm_groups * S, g0 = plan.gh0 * S, g1 = plan.gh1 * S;
      gather(Ly.qkv, tp_rows({{g0, g1}, {kw + g0, kw + g1}, {2 * kw + g0, 2 * kw + g1}}), 0,
             Ly.qkv.nb, Sh.qkv);
      gather(Ly.z, tp_rows({{g0, g1}}), 0, Ly.z.nb, Sh.z);
      gather(Ly.beta, tp_rows({{plan.gh0, plan.gh1}}), 0, Ly.beta.nb, Sh.beta);
      gather(Ly.alpha, tp_rows({{plan.gh0, plan.gh1}}), 0, Ly.alpha.nb, Sh.alpha);
      if (allreduce)
        gather(Ly.out, tp_rows({{0, (int)c.hidden}}), g0 / 256, (g1 - g0) / 256, Sh.out);
      else
        gather(Ly.out, tp_rows({{plan.hr0, plan.hr1}}), 0, Ly.out.nb, Sh.out);
      // convolution weights of this rank's q, k and v channels
      float *cw = nullptr;
      if (e == cudaSuccess) e = batch_alloc(b, &cw, (size_t)3 * (g1 - g0) * c.conv_kernel);
      for (int part = 0; part < 3 && e == cudaSuccess; ++part)
        e = cudaMemcpy(cw + (size_t)part * (g1 - g0) * c.conv_kernel,
                       Ly.conv_w + (size_t)(part * kw + g0) * c.conv_kernel,
                       (size_t)(g1 - g0) * c.conv_kernel * 4, cudaMemcpyDeviceToDevice);
      Sh.conv_w = cw;
      Sh.dt_bias = Ly.dt_bias + plan.gh0;
      Sh.ssm_a = Ly.ssm_a + plan.gh0;
    }
    gather(Ly.up, tp_rows({{plan.fb0 * 256, plan.fb1 * 256}}), 0, Ly.up.nb, Sh.up);
    gather(Ly.gate, tp_rows({{plan.fb0 * 256, plan.fb1 * 256}}), 0, Ly.gate.nb, Sh.gate);
    if (allreduce)
      gather(Ly.down, tp_rows({{0, (int)c.hidden}}), plan.fb0, plan.fb1 - plan.fb0, Sh.down);
    else
      gather(Ly.down, tp_rows({{plan.hr0, plan.hr1}}), 0, Ly.down.nb, Sh.down);
  }
  if (!tpx) {
    b->lm = m->embd;
  } else if (e == cudaSuccess) {
    e = tp_gather_weight(m->embd, tp_rows({{plan.v0, plan.v1}}), 0, m->embd.nb, ex->num_sms,
                         b->allocations, b->stream, b->lm);
  }
#define A(p, n) \
  if (e == cudaSuccess) e = batch_alloc(b, &(p), (n))
  if (!tpx || allreduce) A(b->hidden, B * c.hidden);  // exact: in the exchange buffer
  A(b->xn, B * c.hidden);
  A(b->mixed, B * b->gdn_channels());
  A(b->zgate, B * b->gdn_width());
  A(b->beta, B * b->gdn_heads);
  A(b->alpha, B * b->gdn_heads);
  A(b->attended, B * std::max<size_t>(b->gdn_width(), (size_t)b->heads * hd));
  A(b->projected, B * b->heads * hd * 2);
  A(b->key, B * b->kv_heads * hd);
  A(b->value, B * b->kv_heads * hd);
  A(b->up, B * b->ffn);
  A(b->gate, B * b->ffn);
  uint8_t *tokbuf = nullptr;
  A(tokbuf, token_q8k_bytes(B, (int)std::max<uint32_t>(c.ffn, c.heads * c.head_dim) / 256 + 1));
  b->tok = tokbuf;
  A(b->d_pos, B);
  A(b->d_step, 1);
  A(b->d_tokens, B);
  A(b->d_keys, B);
  for (uint32_t l = 0; l < c.layers; ++l) {
    BatchLayer &Bl = b->L[l];
    if (m->L[l].full) {
      A(Bl.kc, B * b->kv_seq_bytes() / 2);
      A(Bl.vc, B * b->kv_seq_bytes() / 2);
    } else {
      A(Bl.conv, 2 * B * b->gdn_channels() * (c.conv_kernel - 1));
      A(Bl.matrix, B * b->gdn_heads * S * S);
    }
  }
  if (tpx) {
    const int tok_nb = (int)std::max<uint32_t>(std::max<uint32_t>(c.ffn, c.heads * c.head_dim),
                                                (uint32_t)m->value_width()) / 256;
    b->x.layout(allreduce ? kTpAllReduce : kTpExact, plan.size, (int)B, (int)c.hidden, tok_nb);
    A(b->x.base, b->x.bytes);
    A(b->x.xstep, 1);
    if (e == cudaSuccess && !allreduce) b->hidden = b->x.hidden(b->x.base);
  }
#undef A
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    prism_b200_batch_destroy(b);
    return cuda_fail(ex, e, "batch allocation");
  }
  *out = b;
  return PRISM_B200_OK;
}

int prism_b200_tp_plan(const prism_b200_qwen35_config *cfg, uint32_t tp_rank, uint32_t tp_size,
                       int32_t *out) {
  using namespace prism;
  if (!cfg || !out) return PRISM_B200_E_INVALID;
  if (tp_size < 1 || tp_size > (uint32_t)kMaxTp || tp_rank >= tp_size) return PRISM_B200_E_INVALID;
  TpPlan p;
  if (tp_plan(*cfg, (int)tp_rank, (int)tp_size, p)) return PRISM_B200_E_UNSUPPORTED;
  const int32_t v[12] = {p.qh0, p.qh1, p.kv0, p.kv1, p.gh0, p.gh1,
                         p.fb0, p.fb1, p.v0,  p.v1,  p.hr0, p.hr1};
  memcpy(out, v, sizeof(v));
  return PRISM_B200_OK;
}

int prism_b200_batch_exchange_handle(const prism_b200_batch *b, void *handle) {
  if (!b || !handle) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = b->m->ex;
  if (b->tp.size < 2) return ex->fail(PRISM_B200_E_INVALID, "batch is not tensor-parallel");
  cudaSetDevice(ex->device);
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, b->x.base), "exchange handle");
  static_assert(sizeof(h) == PRISM_B200_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return PRISM_B200_OK;
}

int prism_b200_batch_connect(prism_b200_batch *b, const void *handles) {
  using namespace prism;
  if (!b || !handles) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = b->m->ex;
  if (b->tp.size < 2) return ex->fail(PRISM_B200_E_INVALID, "batch is not tensor-parallel");
  if (b->x.connected) return ex->fail(PRISM_B200_E_INVALID, "batch is already connected");
  cudaSetDevice(ex->device);
  const uint8_t *hb = static_cast<const uint8_t *>(handles);
  for (int p = 0; p < b->tp.size; ++p) {
    if (p == b->tp.rank) {
      b->x.peer[p] = b->x.base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)p * sizeof(h), sizeof(h));
    void *ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return ex->fail(PRISM_B200_E_DEVICE, "open rank %d's exchange buffer: %s", p,
                      cudaGetErrorString(e));
    b->x.peer[p] = static_cast<uint8_t *>(ptr);
    b->x.opened[p] = true;
  }
  b->x.connected = true;
  return PRISM_B200_OK;
}

void prism_b200_batch_destroy(prism_b200_batch *b) {
  if (!b) return;
  cudaSetDevice(b->m->ex->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  if (b->graph) cudaGraphExecDestroy(b->graph);
  for (int p = 0; p < prism::kMaxTp; ++p)
    if (b->x.opened[p]) cudaIpcCloseMemHandle(b->x.peer[p]);
  for (void *p : b->allocations) cudaFree(p);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
}

int prism_b200_batch_reset(prism_b200_batch *b) {
  using namespace prism;
  if (!b) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = b->m->ex;
  cudaSetDevice(ex->device);
  const auto &c = b->m->cfg;
  const size_t B = b->B;
  cudaStream_t s = b->stream;
  for (size_t l = 0; l < b->L.size(); ++l) {
    BatchLayer &Bl = b->L[l];
    if (b->m->L[l].full) {
      CK(cudaMemsetAsync(Bl.kc, 0, B * b->kv_seq_bytes(), s), "batch reset");
      CK(cudaMemsetAsync(Bl.vc, 0, B * b->kv_seq_bytes(), s), "batch reset");
    } else {
      CK(cudaMemsetAsync(Bl.conv, 0, 2 * B * b->gdn_channels() * (c.conv_kernel - 1) * 4, s),
         "batch reset");
      CK(cudaMemsetAsync(Bl.matrix, 0, B * b->gdn_heads * c.ssm_state * c.ssm_state * 4, s),
         "batch reset");
    }
  }
  CK(cudaMemsetAsync(b->d_pos, 0, B * 4, s), "batch reset");
  CK(cudaMemsetAsync(b->d_step, 0, 4, s), "batch reset");
  CK(cudaMemsetAsync(b->d_keys, 0, B * 8, s), "batch reset");
  CK(cudaStreamSynchronize(s), "batch reset");
  b->steps = 0;
  return PRISM_B200_OK;
}

static int batch_finish(prism_b200_batch *b) {
  prism_b200_executor *ex = b->m->ex;
  CK(cudaMemcpyAsync(ex->h_status, ex->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost,
                     b->stream),
     "status readback");
  CK(cudaStreamSynchronize(b->stream), "batch step");
  if (*ex->h_status) {
    ex->faulted = true;
    return ex->fail(status_to_code(*ex->h_status), "device reported status 0x%x",
                    *ex->h_status);
  }
  return PRISM_B200_OK;
}

int prism_b200_batch_step(prism_b200_batch *b, const uint32_t *tokens, uint32_t *greedy) {
  using namespace prism;
  if (!b || !tokens) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = b->m->ex;
  int st = check_open(ex);
  if (st) return st;
  const auto &c = b->m->cfg;
  for (int i = 0; i < b->B; ++i)
    if (tokens[i] >= c.vocab) return ex->fail(PRISM_B200_E_INVALID, "token out of range");
  if (b->steps >= b->context) return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  if (b->tp.size > 1 && !b->x.connected)
    return ex->fail(PRISM_B200_E_INVALID, "connect the tensor-parallel ranks first");
  cudaSetDevice(ex->device);
  CK(cudaMemcpyAsync(b->d_tokens, tokens, (size_t)b->B * 4, cudaMemcpyHostToDevice, b->stream),
     "token copy");
  if (!b->graph) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal), "capture");
    cudaError_t e2 = enqueue_batch_step(b, true);
    cudaError_t e = cudaStreamEndCapture(b->stream, &g);
    if (e2 != cudaSuccess) e = e2;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&b->graph, g, 0);
    if (g) cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(ex, e, "batch step capture");
  }
  CK(cudaGraphLaunch(b->graph, b->stream), "batch step");
  if (greedy)
    CK(cudaMemcpyAsync(greedy, b->d_tokens, (size_t)b->B * 4, cudaMemcpyDeviceToHost, b->stream),
       "greedy copy");
  st = batch_finish(b);
  if (st) return st;
  b->steps += 1;
  return PRISM_B200_OK;
}

int prism_b200_batch_decode_async(prism_b200_batch *b, size_t steps) {
  if (!b) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = b->m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!b->graph) return ex->fail(PRISM_B200_E_INVALID, "run one prism_b200_batch_step first");
  cudaSetDevice(ex->device);
  for (size_t i = 0; i < steps; ++i) CK(cudaGraphLaunch(b->graph, b->stream), "batch step");
  b->steps += (int64_t)steps;
  return PRISM_B200_OK;
}

void *prism_b200_batch_stream(const prism_b200_batch *b) {
  return b ? reinterpret_cast<void *>(b->stream) : nullptr;
}

int prism_b200_batch_fill_context(prism_b200_batch *b, uint32_t position, uint64_t seed) {
  using namespace prism;
  if (!b) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = b->m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (position >= (uint32_t)b->context)
    return ex->fail(PRISM_B200_E_INVALID, "position %u outside the context", position);
  cudaSetDevice(ex->device);
  const auto &c = b->m->cfg;
  cudaStream_t s = b->stream;
  const size_t B = b->B;
  for (size_t l = 0; l < b->L.size(); ++l) {
    BatchLayer &Bl = b->L[l];
    const uint64_t ls = seed * 1000003ull + l * 7919ull;
    if (b->m->L[l].full) {
      const long rows = (long)B * b->context;
      const int rb = (int)b->kv_row, q8 = c.kv_policy == PRISM_B200_KV_Q8_0;
      fill_kv_kernel<<<4096, 256, 0, s>>>(reinterpret_cast<uint8_t *>(Bl.kc), rows, rb,
                                          (int)c.head_dim, q8 && b->serve_attn ? 2 : q8,
                                          ls * 2 + 1);
      fill_kv_kernel<<<4096, 256, 0, s>>>(reinterpret_cast<uint8_t *>(Bl.vc), rows, rb,
                                          (int)c.head_dim, q8, ls * 2 + 2);
    } else {
      fill_f32_kernel<<<4096, 256, 0, s>>>(Bl.matrix,
                                           (long)B * b->gdn_heads * c.ssm_state * c.ssm_state,
                                           0.05f, ls * 2 + 3);
      fill_f32_kernel<<<1024, 256, 0, s>>>(Bl.conv,
                                           (long)2 * B * b->gdn_channels() * (c.conv_kernel - 1),
                                           0.5f, ls * 2 + 4);
    }
  }
  std::vector<int> pos(B, (int)position);
  CK(cudaMemcpyAsync(b->d_pos, pos.data(), B * 4, cudaMemcpyHostToDevice, s), "fill");
  CK(cudaGetLastError(), "fill launch");
  CK(cudaStreamSynchronize(s), "fill");
  b->steps = position;
  return PRISM_B200_OK;
}

int64_t prism_b200_batch_read_state(prism_b200_batch *b, uint32_t seq, uint32_t layer,
                                    uint32_t which, void *out, size_t bytes) {
  if (!b || !out || seq >= (uint32_t)b->B) return -PRISM_B200_E_INVALID;
  prism_b200_model *m = b->m;
  const auto &c = m->cfg;
  const void *src = nullptr;
  size_t n = 0;
  if (which == 4) {
    src = b->hidden + (size_t)seq * c.hidden;
    n = (size_t)c.hidden * 4;
  } else if (layer < c.layers) {
    const prism::BatchLayer &Bl = b->L[layer];
    const size_t hist = (size_t)b->gdn_channels() * (c.conv_kernel - 1);
    if (which == 0 && !m->L[layer].full) {
      int step = 0;
      cudaMemcpy(&step, b->d_step, 4, cudaMemcpyDeviceToHost);
      src = Bl.conv + ((size_t)(step & 1) * b->B + seq) * hist;
      n = hist * 4;
    } else if (which == 1 && !m->L[layer].full) {
      const size_t per = (size_t)b->gdn_heads * c.ssm_state * c.ssm_state;
      src = Bl.matrix + seq * per;
      n = per * 4;
    } else if ((which == 2 || which == 3) && m->L[layer].full) {
      int pos = 0;
      cudaMemcpy(&pos, b->d_pos + seq, 4, cudaMemcpyDeviceToHost);
      const uint8_t *base = reinterpret_cast<const uint8_t *>(which == 2 ? Bl.kc : Bl.vc);
      src = base + (size_t)seq * b->kv_seq_bytes();
      n = (size_t)pos * b->kv_row;
      if (b->serve_attn) {
        // head-major cache (K in interleaved pages): rebuild [position][kv head][record]
        if (bytes < n) return -PRISM_B200_E_INVALID;
        const int hd = (int)c.head_dim, rb = prism::q8_0_record_bytes(hd);
        std::vector<uint8_t> head((size_t)b->context * rb);
        uint8_t *dst = static_cast<uint8_t *>(out);
        cudaSetDevice(m->ex->device);
        const uint32_t kvh = (uint32_t)b->kv_heads;
        for (uint32_t k = 0; k < kvh && pos > 0; ++k) {
          if (cudaMemcpy(head.data(), static_cast<const uint8_t *>(src) + (size_t)k * b->context * rb,
                         head.size(), cudaMemcpyDeviceToHost) != cudaSuccess)
            return -PRISM_B200_E_DEVICE;
          for (int p = 0; p < pos; ++p) {
            uint8_t *rec = dst + ((size_t)p * kvh + k) * rb;
            if (which == 3) {
              memcpy(rec, head.data() + (size_t)p * rb, rb);
              continue;
            }
            const uint8_t *page = head.data() + (size_t)(p / prism::kServePage) * prism::kServePage * rb;
            const int slot = p % prism::kServePage;
            for (int blk = 0; blk < hd / 32; ++blk)
              memcpy(rec + 2 * blk, page + prism::kpage_scale(hd, blk, slot), 2);
            for (int d = 0; d < hd; ++d) rec[hd / 32 * 2 + d] = page[prism::kpage_code(hd, d, slot)];
          }
        }
        return (int64_t)n;
      }
    }
  }
  if (!src) return -PRISM_B200_E_INVALID;
  if (bytes < n) return -PRISM_B200_E_INVALID;
  cudaSetDevice(m->ex->device);
  if (cudaMemcpyAsync(out, src, n, cudaMemcpyDeviceToHost, b->stream) != cudaSuccess ||
      cudaStreamSynchronize(b->stream) != cudaSuccess)
    return -PRISM_B200_E_DEVICE;
  return (int64_t)n;
}

}  // extern "C"
