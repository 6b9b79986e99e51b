// model.cuh -- C ABI of the Qwen3.5-style hybrid decoder on the device.
//
// Included once by prism_b200.cu (one translation unit owns every kernel).
// One decode step is a fixed sequence of launches on the model's stream,
// captured once into a CUDA graph and replayed per token.  All step state
// (position, token history, greedy key) lives in device memory, so a graph
// replay needs no host input and consecutive replays generate greedily
// without returning to the host.  Launches use programmatic dependent
// launch, so each projection streams its weights while the previous kernel
// finishes.
#pragma once

#include <atomic>
#include <map>
#include <string>
#include <vector>

#include "executor.cuh"
#include "flow.cuh"
#include "model_kernels.cuh"
#include "kvq.cuh"
#include "gdn_decode.cuh"

namespace prism {

struct ModelLayer {
  bool full = false;
  DeviceWeight gate, up, down;
  DeviceWeight q, k, v, o;                   // full attention
  DeviceWeight qkv, z, beta, alpha, out;     // Gated DeltaNet
  float *attn_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  float *conv_w = nullptr, *dt_bias = nullptr, *ssm_a = nullptr, *ssm_norm = nullptr;
  float *conv_state = nullptr;   // 2 x [channels][k-1]
  float *matrix = nullptr;       // [values][S][S]
  uint16_t *kc = nullptr, *vc = nullptr;  // [context][kv*hd]
};

// Activations of the batched prompt pass (prefill.cuh), [kPrefillChunk]
// tokens each, allocated on its first use.
struct PrefillBuffers {
  float *hidden = nullptr, *xn = nullptr, *mixed = nullptr, *zgate = nullptr, *beta = nullptr,
        *alpha = nullptr, *o_pre = nullptr, *attended = nullptr, *projected = nullptr,
        *key = nullptr, *value = nullptr, *up = nullptr, *gate = nullptr, *act = nullptr,
        *db = nullptr;
  float *qrows = nullptr, *scur = nullptr, *scratch = nullptr;  // batched attention
  void *tok = nullptr;  // Q8_K tokens of the widest projection input
  int *pos = nullptr;   // position of each token
  bool ready = false;
};

}  // namespace prism

struct prism_b200_model {
  prism_b200_executor *ex = nullptr;
  uint64_t serial = 0;  // process-unique: the provenance a checkpoint carries
  prism_b200_qwen35_config cfg{};
  std::vector<prism::ModelLayer> L;
  prism::DeviceWeight embd;
  float *out_norm = nullptr;
  // activations
  float *hidden = nullptr, *mixed = nullptr, *zgate = nullptr, *beta = nullptr, *alpha = nullptr;
  float *attended = nullptr, *projected = nullptr, *key = nullptr, *value = nullptr;
  float *up = nullptr, *gatef = nullptr, *logits = nullptr;
  // step state
  int *d_position = nullptr;
  uint32_t *d_tokens = nullptr;
  int *d_prompt_end = nullptr;
  unsigned long long *d_argmax = nullptr;
  int64_t position = 0;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t g_ingest = nullptr, g_decode = nullptr;
  // per-kernel timelines of the kernel-sequence step (PRISM_B200_TRACE=1 set
  // before finalize): [8 * launches], projection / GDN / attention launches
  unsigned long long *d_seqtrace = nullptr;
  int nseqtrace = 0;
  float *gdn_o = nullptr;
  // the dataflow step (flow.cuh): phase list, tagged activations, step words
  bool flow = false;
  prism::FPhase *d_fphases = nullptr;
  int nfphases = 0;
  unsigned *d_fsync = nullptr;  // [0] finished CTAs, [1] abort, [2] step epoch
  unsigned long long *d_fkey = nullptr;  // greedy key while a dataflow step runs
  unsigned long long *d_ftrace = nullptr, *d_ftrace_cta = nullptr;
  uint64_t *t_hidden = nullptr, *t_mixed = nullptr, *t_z = nullptr, *t_beta = nullptr,
           *t_alpha = nullptr, *t_o = nullptr, *t_zs = nullptr, *t_proj = nullptr,
           *t_key = nullptr, *t_value = nullptr, *t_att = nullptr, *t_up = nullptr,
           *t_scores = nullptr;
  prism::PrefillBuffers pre;
  std::map<std::string, bool> bound;
  std::vector<void *> allocations;
  bool finalized = false;

  int key_width() const { return (int)(cfg.ssm_state * cfg.ssm_groups); }
  int value_width() const { return (int)(cfg.ssm_state * cfg.ssm_values); }
  int channels() const { return 2 * key_width() + value_width(); }
  int kvw() const { return (int)(cfg.kv_heads * cfg.head_dim); }
  // the reference's rotated scalar records (rsq4, rsq4vf, rsq4k3v)
  bool rotated() const { return cfg.kv_policy >= PRISM_B200_KV_RSQ4; }
  int value_bits() const { return cfg.kv_policy == PRISM_B200_KV_RSQ4K3V ? 3 : 4; }
  // bytes of one cached position (all KV heads) of one layer's K or V
  size_t kv_row_bytes(bool value = false) const {
    if (rotated())
      return (size_t)cfg.kv_heads * prism::kvq_record_bytes(value ? value_bits() : 4);
    return cfg.kv_policy == PRISM_B200_KV_Q8_0
               ? (size_t)cfg.kv_heads * prism::q8_0_record_bytes((int)cfg.head_dim)
               : (size_t)kvw() * 2;
  }
  bool is_full(int l) const { return ((l + 1) % (int)cfg.full_interval) == 0; }
};

namespace prism {

// The step mode: the dataflow step (2) where the model and device are
// eligible, else the kernel sequence (0); PRISM_B200_STEP=seq selects the
// kernel sequence.
inline int step_mode_request() {
  const char *e = getenv("PRISM_B200_STEP");
  return e && !strcmp(e, "seq") ? 0 : 2;
}

// Dynamic shared memory of an attention_decode_kernel launch over a cache of
// `context` positions: with the CTA's K and V rows staged when they fit
// (sets a.kv_smem_off), else the in-place layout.
inline size_t attn_launch_smem(AttnArgs &a, int context) {
  static const bool stage_on = [] {
    const char *e = getenv("PRISM_B200_ATTN_STAGE");  // 0: read rows in place (A/B timing)
    return !(e && e[0] == '0');
  }();
  const size_t staged = attn_smem_bytes_staged(a.hd, context, a.q8);
  if (stage_on && staged <= (size_t)kMaxSmem &&
      cudaFuncSetAttribute(attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)staged) == cudaSuccess) {
    a.kv_smem_off = (int)attn_smem_bytes(a.hd, context);
    return staged;
  }
  a.kv_smem_off = 0;
  return attn_smem_bytes(a.hd, context);
}

template <typename T>
cudaError_t model_alloc(prism_b200_model *m, T **p, size_t count) {
  void *v = nullptr;
  cudaError_t e = cudaMalloc(&v, count * sizeof(T) < 16 ? 16 : count * sizeof(T));
  if (e != cudaSuccess) return e;
  e = cudaMemset(v, 0, count * sizeof(T) < 16 ? 16 : count * sizeof(T));
  m->allocations.push_back(v);
  *p = static_cast<T *>(v);
  return e;
}

inline StepState step_state(prism_b200_model *m) {
  StepState st;
  st.position = m->d_position;
  st.tokens = m->d_tokens;
  st.prompt_end = m->d_prompt_end;
  st.argmax = m->d_argmax;
  return st;
}

// The step's launches in order (projection groups, Gated DeltaNet,
// attention; the LM head last with `head`), each with the HBM ranges it
// reads that no earlier kernel of the step writes: weights and recurrent
// state.  Projection launches prefetch these into L2 a few launches ahead
// (kPrefetchAhead), so the weight stream runs under the dependent chain of
// small kernels instead of inside it; the last launches of a step prefetch
// the first ones of the next step (the same weights).
constexpr int kPrefetchAhead = 3;
constexpr size_t kPrefetchCap = 24u << 20;  // bytes of one range (the LM head's first part)

struct PfItem {
  std::vector<std::pair<const uint8_t *, size_t>> r;
  void add(const void *p, size_t bytes) {
    if (p && bytes) r.emplace_back(static_cast<const uint8_t *>(p), std::min(bytes, kPrefetchCap) / 16 * 16);
  }
  void add(const DeviceWeight &w) { add(w.units, w.bytes); }
};

inline std::vector<PfItem> step_items(prism_b200_model *m, bool head) {
  const auto &c = m->cfg;
  std::vector<PfItem> items;
  for (const ModelLayer &Ly : m->L) {
    PfItem g, mid, out, ffn, down;
    if (Ly.full) {
      g.add(Ly.q);
      g.add(Ly.k);
      g.add(Ly.v);
      out.add(Ly.o);
    } else {
      g.add(Ly.qkv);
      g.add(Ly.z);
      g.add(Ly.beta);
      g.add(Ly.alpha);
      mid.add(Ly.matrix, (size_t)c.ssm_values * c.ssm_state * c.ssm_state * 4);
      mid.add(Ly.conv_state, (size_t)2 * m->channels() * (c.conv_kernel - 1) * 4);
      out.add(Ly.out);
    }
    ffn.add(Ly.up);
    ffn.add(Ly.gate);
    down.add(Ly.down);
    items.push_back(g);
    items.push_back(mid);
    items.push_back(out);
    items.push_back(ffn);
    items.push_back(down);
  }
  if (head) {
    PfItem h;
    h.add(m->embd);
    items.push_back(h);
  }
  return items;
}

// The attention of a full layer over rotated scalar records (kv_policy
// rsq4, rsq4vf, rsq4k3v; reference src/graph/quantized_kv.rs:16-84): the
// append kernel encodes the current key and value rows at the step's
// position, then kvq_attend_kernel attends over every record.
inline cudaError_t launch_kvq_step(prism_b200_model *m, const ModelLayer &Ly, unsigned *status,
                                   cudaStream_t s, bool pdl) {
  const auto &c = m->cfg;
  const int vbits = m->value_bits();
  static const KvqCodec kc = kvq_codec(4, kKvqKeySeed, 1);
  const KvqCodec vc = kvq_codec(vbits, kKvqValueSeed, c.kv_policy == PRISM_B200_KV_RSQ4VF ? 2 : 1);
  const float theta_scale = powf(c.rope_base, -2.0f / (float)c.rope_dim);
  KvqAppendArgs ap{};
  ap.kc = kc;
  ap.vc = vc;
  ap.kv_heads = (int)c.kv_heads;
  ap.rope_dim = (int)c.rope_dim;
  for (int j = 0; j < 3; ++j) ap.sections[j] = (int)c.rope_sections[j];
  ap.eps = c.eps;
  ap.theta_scale = theta_scale;
  ap.key_in = m->key;
  ap.value_in = m->value;
  ap.k_norm = Ly.k_norm;
  ap.kcache = reinterpret_cast<uint8_t *>(Ly.kc);
  ap.vcache = reinterpret_cast<uint8_t *>(Ly.vc);
  ap.position = m->d_position;
  ap.status = status;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(2 * c.kv_heads), dim3(kKvqDim), 0, s, attr, pdl);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kvq_append_kernel, ap);
  if (e != cudaSuccess) return e;
  KvqAttnArgs at{};
  at.kc = kc;
  at.vc = vc;
  at.heads = (int)c.heads;
  at.kv_heads = (int)c.kv_heads;
  at.projected = m->projected;
  at.q_norm = Ly.q_norm;
  at.eps = c.eps;
  at.theta_scale = theta_scale;
  at.rope_dim = (int)c.rope_dim;
  for (int j = 0; j < 3; ++j) at.sections[j] = (int)c.rope_sections[j];
  at.gate = m->projected + kKvqDim;  // head h's gate row follows its query row
  at.gate_stride = 2 * kKvqDim;
  at.keys = ap.kcache;
  at.values = ap.vcache;
  at.position = m->d_position;
  at.attn_scale = 1.0f / 16.0f;  // 1 / sqrt(256)
  at.out = m->attended;
  at.status = status;
  return launch_kvq_attend(at, (int)c.context, s, pdl);
}

// Enqueue one decode step.  With `head`, the step ends with the tied LM head,
// the greedy key and (past the prompt) the next input token.
// `ev` (optional, 2*layers + 4 events) brackets the phases for per-layer
// timing: ev[0] start, ev[1] after the embedding, ev[2+2l] after layer l's
// attention, ev[3+2l] after its FFN, ev[2+2L] after the head, ev[3+2L] end.
// Timed steps run without programmatic dependent launch.
inline cudaError_t enqueue_step(prism_b200_model *m, bool head, cudaEvent_t *ev = nullptr) {
  prism_b200_executor *ex = m->ex;
  const auto &c = m->cfg;
  const bool pdl = ex->pdl && !ev;
  const int nl = (int)m->L.size();
  auto mark = [&](int i) {
    if (ev) cudaEventRecord(ev[i], m->stream);
  };
  mark(0);
  const int sms = ex->num_sms;
  cudaStream_t s = m->stream;
  unsigned *status = ex->d_status;
  cudaLaunchAttribute attr[1];
  cudaError_t e;
  {
    const int n = (int)c.hidden;
    cudaLaunchConfig_t cfg = pdl_config(dim3((n + 255) / 256), dim3(256), 0, s, attr, pdl);
    const uint8_t *units = m->embd.units;
    const int h = m->embd.h, nb = m->embd.nb, vocab = (int)c.vocab;
    float *hidden = m->hidden;
    e = c.weight_kind == 35
            ? cudaLaunchKernelEx(&cfg, embed_kernel<35>, units, h, nb, vocab, step_state(m),
                                 hidden, n, status)
            : cudaLaunchKernelEx(&cfg, embed_kernel<10>, units, h, nb, vocab, step_state(m),
                                 hidden, n, status);
    if (e != cudaSuccess) return e;
  }
  mark(1);
  const uint32_t kind = c.weight_kind;
  // L2 prefetch: launch `item` covers the items after `horizon` up to
  // item + kPrefetchAhead (wrapping into the next step)
  const std::vector<PfItem> items = step_items(m, head);
  const int nitems = (int)items.size();
  int item = 0, horizon = kPrefetchAhead;  // the first items are the previous step's
  static const bool pf_on = [] {
    const char *e = getenv("PRISM_B200_PREFETCH");  // 0: off (A/B timing)
    return !(e && e[0] == '0');
  }();
  auto prefetch = [&](MvArgs &a) {
    if (!pf_on) return;
    int k = 0;
    for (; horizon < item + kPrefetchAhead; ++horizon) {
      for (const auto &r : items[(horizon + 1) % nitems].r)
        if (k < kMaxPrefetch) {
          a.pf[k] = r.first;
          a.pf_bytes[k] = (unsigned)r.second;
          ++k;
        }
    }
  };
  // optional per-launch timelines (not on event-timed steps)
  auto trace_slot = [&]() -> unsigned long long * {
    return m->d_seqtrace && !ev && item < m->nseqtrace ? m->d_seqtrace + 8 * item : nullptr;
  };
  if (m->d_seqtrace && !ev) {
    if ((e = cudaMemsetAsync(m->d_seqtrace, 0, (size_t)64 * m->nseqtrace, s)) != cudaSuccess)
      return e;
  }
  auto launch_mv = [&](int epi, MvArgs &a) {
    prefetch(a);
    a.trace = trace_slot();
    ++item;
    return launch_matvec_group(kind, epi, a, sms, s, pdl);
  };
  for (size_t l = 0; l < m->L.size(); ++l) {
    ModelLayer &Ly = m->L[l];
    MvArgs a;
    a.prologue = kProRmsNorm;
    a.in0 = m->hidden;
    a.norm_w = Ly.attn_norm;
    a.eps = c.eps;
    a.status = status;
    a.nb = (int)(c.hidden / 256);
    if (Ly.full) {
      a.count = 3;
      a.w[0] = mv_weight(Ly.q, m->projected);
      a.w[1] = mv_weight(Ly.k, m->key);
      a.w[2] = mv_weight(Ly.v, m->value);
      if ((e = launch_mv(kEpiStore, a)) != cudaSuccess) return e;
      if (m->rotated()) {
        // the reference's rotated scalar records: encode the current K/V
        // rows, then attend over every record
        if ((e = launch_kvq_step(m, Ly, status, s, pdl)) != cudaSuccess) return e;
        ++item;
      } else {
        AttnArgs aa{};
        aa.heads = (int)c.heads;
        aa.kv_heads = (int)c.kv_heads;
        aa.hd = (int)c.head_dim;
        aa.rope_dim = (int)c.rope_dim;
        for (int j = 0; j < 3; ++j) aa.sections[j] = (int)c.rope_sections[j];
        aa.eps = c.eps;
        aa.theta_scale = powf(c.rope_base, -2.0f / (float)c.rope_dim);
        aa.projected = m->projected;
        aa.key_in = m->key;
        aa.value_in = m->value;
        aa.q_norm = Ly.q_norm;
        aa.k_norm = Ly.k_norm;
        aa.kcache = Ly.kc;
        aa.vcache = Ly.vc;
        aa.q8 = c.kv_policy == PRISM_B200_KV_Q8_0 ? 1 : 0;
        aa.position = m->d_position;
        aa.attended = m->attended;
        aa.status = status;
        aa.trace = trace_slot();
        // one 8-CTA cluster per query head (split over the cached positions)
        const size_t smem = attn_launch_smem(aa, (int)c.context);
        cudaLaunchAttribute cattr[2];
        cudaLaunchConfig_t cfg = pdl_config(dim3(c.heads * kAttnSplit), dim3(kAttnThreads), smem,
                                            s, cattr, pdl);
        cattr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        cattr[cfg.numAttrs].val.clusterDim.x = kAttnSplit;
        cattr[cfg.numAttrs].val.clusterDim.y = 1;
        cattr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs += 1;
        if ((e = cudaLaunchKernelEx(&cfg, attention_decode_kernel, aa)) != cudaSuccess) return e;
        ++item;
      }
      MvArgs o;
      o.prologue = kProF32;
      o.in0 = m->attended;
      o.status = status;
      o.nb = (int)(c.heads * c.head_dim / 256);
      o.count = 1;
      o.w[0] = mv_weight(Ly.o, m->hidden, m->hidden);
      if ((e = launch_mv(kEpiStore, o)) != cudaSuccess) return e;
    } else {
      a.count = 4;
      a.w[0] = mv_weight(Ly.qkv, m->mixed);
      a.w[1] = mv_weight(Ly.z, m->zgate);
      a.w[2] = mv_weight(Ly.beta, m->beta);
      a.w[3] = mv_weight(Ly.alpha, m->alpha);
      if ((e = launch_mv(kEpiStore, a)) != cudaSuccess) return e;
      GdnArgs g;
      g.trace = trace_slot();
      g.S = (int)c.ssm_state;
      g.groups = (int)c.ssm_groups;
      g.values = (int)c.ssm_values;
      g.conv_k = (int)c.conv_kernel;
      g.eps = c.eps;
      g.mixed = m->mixed;
      g.zgate = m->zgate;
      g.beta_in = m->beta;
      g.alpha_in = m->alpha;
      g.in_stride = g.z_stride = g.ab_stride = 0;
      g.conv_w = Ly.conv_w;
      g.dt_bias = Ly.dt_bias;
      g.ssm_a = Ly.ssm_a;
      g.norm_w = Ly.ssm_norm;
      g.conv_state = Ly.conv_state;
      g.conv_buf_stride = (long)m->channels() * (c.conv_kernel - 1);
      g.conv_stride = 0;
      g.state = Ly.matrix;
      g.state_stride = 0;
      g.attended = m->gdn_o;  // pre-norm o; the gated norm is the out-projection's prologue
      g.out_stride = 0;
      g.position = m->d_position;
      g.status = status;
      // each value head over kGdnSlices CTAs of 16 state rows
      cudaLaunchConfig_t cfg =
          pdl_config(dim3(c.ssm_values * kGdnSlices), dim3(kGdnThreads), 0, s, attr, pdl);
      if ((e = cudaLaunchKernelEx(&cfg, gdn_slices_kernel, g)) != cudaSuccess) return e;
      ++item;
      MvArgs o;
      o.prologue = kProGated;
      o.in0 = m->gdn_o;
      o.zgate = m->zgate;  // SiLU(z) after the GDN kernel
      o.norm_w = Ly.ssm_norm;
      o.gheads = (int)c.ssm_values;
      o.ghd = (int)c.ssm_state;
      o.eps = c.eps;
      o.status = status;
      o.nb = m->value_width() / 256;
      o.count = 1;
      o.w[0] = mv_weight(Ly.out, m->hidden, m->hidden);
      if ((e = launch_mv(kEpiStore, o)) != cudaSuccess) return e;
    }
    mark(2 + 2 * (int)l);
    MvArgs f;
    f.prologue = kProRmsNorm;
    f.in0 = m->hidden;
    f.norm_w = Ly.post_norm;
    f.eps = c.eps;
    f.status = status;
    f.nb = (int)(c.hidden / 256);
    f.count = 2;
    f.w[0] = mv_weight(Ly.up, m->up);  // receives up * silu(gate)
    f.w[1] = mv_weight(Ly.gate, nullptr);
    if ((e = launch_mv(kEpiSwiglu, f)) != cudaSuccess) return e;
    MvArgs d;
    d.prologue = kProF32;
    d.in0 = m->up;
    d.status = status;
    d.nb = (int)(c.ffn / 256);
    d.count = 1;
    d.w[0] = mv_weight(Ly.down, m->hidden, m->hidden);
    if ((e = launch_mv(kEpiStore, d)) != cudaSuccess) return e;
    mark(3 + 2 * (int)l);
  }
  if (head) {
    MvArgs h;
    h.prologue = kProRmsNorm;
    h.in0 = m->hidden;
    h.norm_w = m->out_norm;
    h.eps = c.eps;
    h.status = status;
    h.nb = (int)(c.hidden / 256);
    h.count = 1;
    h.w[0] = mv_weight(m->embd, m->logits);
    h.argmax_key = m->d_argmax;
    if ((e = launch_mv(kEpiArgmax, h)) != cudaSuccess) return e;
  }
  mark(2 + 2 * nl);
  cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(32), 0, s, attr, pdl);
  e = cudaLaunchKernelEx(&cfg, finish_step_kernel, step_state(m), head ? 1 : 0);
  mark(3 + 2 * nl);
  return e;
}

// ---- the dataflow step (flow.cuh) ---------------------------------------------

// The step's phases in order; phase k writes its outputs with tag k, and each
// reader names the phase that wrote its input.  The ingest list stops before
// the LM head (the last phase).
inline std::vector<FPhase> build_flow_phases(prism_b200_model *m) {
  const auto &c = m->cfg;
  std::vector<FPhase> P;
  auto proj = [&](int prologue, const uint64_t *in, int in_k, const float *norm_w, int nb,
                  std::initializer_list<std::pair<const DeviceWeight *, uint64_t *>> ws,
                  int epi) {
    FPhase ph;
    memset(&ph, 0, sizeof(ph));
    ph.type = kFProj;
    ph.k = (int)P.size();
    FProj &pr = ph.pr;
    pr.prologue = prologue;
    pr.in = in;
    pr.in_k = in_k;
    pr.norm_w = norm_w;
    pr.eps = c.eps;
    pr.nb = nb;
    pr.epi = epi;
    pr.count = 0;
    for (const auto &w : ws) {
      const int g = pr.count++;
      pr.units[g] = w.first->units;
      pr.h[g] = w.first->h;
      pr.rows[g] = (int)w.first->rows;
      pr.out[g] = w.second;
      pr.tile_start[g + 1] = pr.tile_start[g] + w.first->ntiles;
    }
    for (int g = pr.count; g < kMaxGroup; ++g) pr.tile_start[g + 1] = pr.tile_start[pr.count];
    pr.ntiles = epi == kEpiSwiglu ? ws.begin()->first->ntiles : pr.tile_start[pr.count];
    // weight-stream pieces: runs of about kFPieceMax bytes, one tile at
    // least, no more tiles than a batch holds (a warp per tile; terms fit)
    const bool pair = epi == kEpiSwiglu;
    const int upt = pair ? 2 * nb : nb;
    const int tiles = std::min(kFWarps, (kFWorkBytes / 4) / (upt * 32));
    for (int g = 0; g < pr.count; ++g) {
      pr.part[g] = nb * unit_bytes((int)c.weight_kind, pr.h[g]);
      const int per = pair ? 2 * pr.part[g] : pr.part[g];
      pr.most[g] = std::max(1, std::min(tiles, kFPieceMax / per));
    }
    return ph;
  };
  int k_hidden = 0;
  {
    FPhase ph;
    memset(&ph, 0, sizeof(ph));
    ph.type = kFEmbed;
    ph.k = 0;
    ph.em.units = m->embd.units;
    ph.em.h = m->embd.h;
    ph.em.nb = m->embd.nb;
    ph.em.vocab = (int)c.vocab;
    ph.em.n = (int)c.hidden;
    ph.em.hidden = m->t_hidden;
    ph.em.plain = m->hidden;
    P.push_back(ph);
  }
  const int hnb = (int)(c.hidden / 256);
  for (auto &Ly : m->L) {
    if (Ly.full) {
      FPhase a1 = proj(kFRms, m->t_hidden, k_hidden, Ly.attn_norm, hnb,
                       {{&Ly.q, m->t_proj}, {&Ly.k, m->t_key}, {&Ly.v, m->t_value}}, kEpiStore);
      P.push_back(a1);
      FPhase ph;
      memset(&ph, 0, sizeof(ph));
      ph.type = kFAttn;
      ph.k = (int)P.size();
      FAttn &at = ph.at;
      at.proj = m->t_proj;
      at.key = m->t_key;
      at.value = m->t_value;
      at.in_k = a1.k;
      at.q_norm = Ly.q_norm;
      at.k_norm = Ly.k_norm;
      at.kcache = reinterpret_cast<uint8_t *>(Ly.kc);
      at.vcache = reinterpret_cast<uint8_t *>(Ly.vc);
      at.q8 = c.kv_policy == PRISM_B200_KV_Q8_0 ? 1 : 0;
      at.heads = (int)c.heads;
      at.kv_heads = (int)c.kv_heads;
      at.hd = (int)c.head_dim;
      at.rope_dim = (int)c.rope_dim;
      for (int j = 0; j < 3; ++j) at.sections[j] = (int)c.rope_sections[j];
      at.eps = c.eps;
      at.theta_scale = powf(c.rope_base, -2.0f / (float)c.rope_dim);
      at.sc = m->t_scores;
      at.ctx = (int)c.context;
      at.out = m->t_att;
      P.push_back(ph);
      FPhase a3 = proj(kFF32, m->t_att, ph.k, nullptr, (int)(c.heads * c.head_dim / 256),
                       {{&Ly.o, m->t_hidden}}, kEpiStore);
      a3.pr.res = m->t_hidden;
      a3.pr.res_k = k_hidden;
      a3.pr.plain[0] = m->hidden;
      P.push_back(a3);
      k_hidden = a3.k;
    } else {
      FPhase g1 = proj(kFRms, m->t_hidden, k_hidden, Ly.attn_norm, hnb,
                       {{&Ly.qkv, m->t_mixed}, {&Ly.z, m->t_z}, {&Ly.beta, m->t_beta},
                        {&Ly.alpha, m->t_alpha}},
                       kEpiStore);
      P.push_back(g1);
      FPhase ph;
      memset(&ph, 0, sizeof(ph));
      ph.type = kFGdn;
      ph.k = (int)P.size();
      FGdn &g = ph.gd;
      g.mixed = m->t_mixed;
      g.z = m->t_z;
      g.beta = m->t_beta;
      g.alpha = m->t_alpha;
      g.in_k = g1.k;
      g.conv_w = Ly.conv_w;
      g.dt_bias = Ly.dt_bias;
      g.ssm_a = Ly.ssm_a;
      g.conv_state = Ly.conv_state;
      g.conv_buf_stride = (long)m->channels() * (c.conv_kernel - 1);
      g.state = Ly.matrix;
      g.o = m->t_o;
      g.zs = m->t_zs;
      g.S = (int)c.ssm_state;
      g.groups = (int)c.ssm_groups;
      g.values = (int)c.ssm_values;
      g.conv_k = (int)c.conv_kernel;
      g.eps = c.eps;
      P.push_back(ph);
      FPhase g3 = proj(kFGated, m->t_o, ph.k, Ly.ssm_norm, m->value_width() / 256,
                       {{&Ly.out, m->t_hidden}}, kEpiStore);
      g3.pr.zs = m->t_zs;
      g3.pr.zs_k = ph.k;
      g3.pr.heads = (int)c.ssm_values;
      g3.pr.head_dim = (int)c.ssm_state;
      g3.pr.res = m->t_hidden;
      g3.pr.res_k = k_hidden;
      g3.pr.plain[0] = m->hidden;
      P.push_back(g3);
      k_hidden = g3.k;
    }
    FPhase f1 = proj(kFRms, m->t_hidden, k_hidden, Ly.post_norm, hnb,
                     {{&Ly.up, m->t_up}, {&Ly.gate, nullptr}}, kEpiSwiglu);
    P.push_back(f1);
    FPhase f2 = proj(kFF32, m->t_up, f1.k, nullptr, (int)(c.ffn / 256), {{&Ly.down, m->t_hidden}},
                     kEpiStore);
    f2.pr.res = m->t_hidden;
    f2.pr.res_k = k_hidden;
    f2.pr.plain[0] = m->hidden;
    P.push_back(f2);
    k_hidden = f2.k;
  }
  FPhase hd = proj(kFRms, m->t_hidden, k_hidden, m->out_norm, hnb, {{&m->embd, nullptr}},
                   kEpiArgmax);
  hd.pr.plain[0] = m->logits;
  hd.pr.argmax_key = m->d_fkey;
  P.push_back(hd);
  return P;
}

// Whether this model and device fit the dataflow step's fixed limits.
inline bool flow_eligible(prism_b200_model *m, const std::vector<FPhase> &P) {
  const auto &c = m->cfg;
  const int sms = m->ex->num_sms;
  int coop = 0, optin = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->ex->device);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->ex->device);
  if (!coop || optin < kFSmemBytes) return false;
  if ((int)(c.heads * kAttnSplit) > sms || (int)(c.ssm_values * kGdnSlices) > sms) return false;
  if (c.ssm_state != 128 || c.head_dim != 256 || c.conv_kernel > 8) return false;
  if (c.context > (uint32_t)kFAttnMaxPos) return false;
  if (m->rotated()) return false;  // rotated records: the kernel sequence
  if (P.size() > 255) return false;  // the phase index is an 8-bit tag field
  for (const FPhase &ph : P) {
    if (ph.type != kFProj) continue;
    const FProj &pr = ph.pr;
    if (pr.nb > kFMaxNb) return false;
    if (pr.epi == kEpiSwiglu && pr.h[0] != pr.h[1]) return false;
    for (int g = 0; g < pr.count; ++g) {
      const long piece = (long)pr.nb * unit_bytes((int)c.weight_kind, pr.h[g]) *
                         (pr.epi == kEpiSwiglu ? 2 : 1);
      if (piece > kFRing / 3) return false;
    }
    // one tile's terms must fit the work area; a CTA's pieces fit its list
    if ((pr.epi == kEpiSwiglu ? 2 : 1) * pr.nb * 32 * 4 > kFWorkBytes) return false;
    if ((pr.ntiles + sms - 1) / sms + pr.count > kFMaxPieces) return false;
  }
  int blocks = 0;
  void *k = c.weight_kind == 35 ? (void *)decode_flow_kernel<35> : (void *)decode_flow_kernel<10>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmemBytes) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, kFBlock, kFSmemBytes) !=
          cudaSuccess ||
      blocks < 1)
    return false;
  return true;
}

inline cudaError_t prepare_flow(prism_b200_model *m) {
  m->flow = false;
  if (step_mode_request() != 2) return cudaSuccess;
  std::vector<FPhase> P = build_flow_phases(m);
  if (!flow_eligible(m, P)) return cudaSuccess;
  if (!m->d_fphases) {
    // a model's layer count, and so its phase count, is fixed at creation
    cudaError_t e = model_alloc(m, &m->d_fphases, P.size());
    if (e == cudaSuccess) e = model_alloc(m, &m->d_ftrace, 16 * P.size());
    if (e == cudaSuccess)
      e = model_alloc(m, &m->d_ftrace_cta, (size_t)4 * m->ex->num_sms * P.size());
    if (e != cudaSuccess) return e;
  }
  m->nfphases = (int)P.size();
  cudaError_t e = cudaMemcpy(m->d_fphases, P.data(), P.size() * sizeof(FPhase),
                             cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return e;
  m->flow = true;
  return cudaSuccess;
}

// One cooperative launch: the whole step (with the LM head when `head`).
inline cudaError_t launch_flow(prism_b200_model *m, bool head, bool trace = false) {
  FlowArgs fa;
  fa.phases = m->d_fphases;
  fa.nphases = head ? m->nfphases : m->nfphases - 1;
  fa.st = step_state(m);
  fa.write_greedy = head ? 1 : 0;
  fa.sync = m->d_fsync;
  fa.key = m->d_fkey;
  fa.status = m->ex->d_status;
  fa.trace = trace ? m->d_ftrace : nullptr;
  fa.trace_cta = trace ? m->d_ftrace_cta : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)m->ex->num_sms);
  cfg.blockDim = dim3(kFBlock);
  cfg.dynamicSmemBytes = kFSmemBytes;
  cfg.stream = m->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return m->cfg.weight_kind == 35 ? cudaLaunchKernelEx(&cfg, decode_flow_kernel<35>, fa)
                                  : cudaLaunchKernelEx(&cfg, decode_flow_kernel<10>, fa);
}

inline cudaError_t capture_step(prism_b200_model *m, bool head, cudaGraphExec_t *out) {
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return e;
  cudaError_t e2 = m->flow ? launch_flow(m, head) : enqueue_step(m, head);
  e = cudaStreamEndCapture(m->stream, &graph);
  if (e2 != cudaSuccess) e = e2;
  if (e == cudaSuccess) e = cudaGraphInstantiate(out, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  return e;
}

// Parse "blk.N.suffix" -> (N, suffix); returns -1 for global names.
inline int parse_layer(const char *name, std::string &suffix) {
  std::string s(name);
  if (s.rfind("blk.", 0) != 0) {
    suffix = s;
    return -1;
  }
  size_t dot = s.find('.', 4);
  if (dot == std::string::npos) return -2;
  int l = atoi(s.substr(4, dot - 4).c_str());
  suffix = s.substr(dot + 1);
  return l;
}

}  // namespace prism

extern "C" {

int prism_b200_model_create(prism_b200_executor *ex, const prism_b200_qwen35_config *cfg,
                            prism_b200_model **out) {
  using namespace prism;
  if (!ex || !cfg || !out) return PRISM_B200_E_INVALID;
  *out = nullptr;
  const auto &c = *cfg;
  const bool ok =
      c.hidden % 256 == 0 && c.hidden > 0 && c.layers > 0 && c.heads > 0 && c.kv_heads > 0 &&
      c.heads % c.kv_heads == 0 && c.head_dim == 256 && c.rope_dim <= c.head_dim &&
      c.rope_dim % 2 == 0 && c.rope_dim <= 64 && c.ffn % 256 == 0 && c.ffn > 0 && c.vocab > 0 &&
      c.ssm_state == 128 && c.ssm_groups > 0 && c.ssm_values % c.ssm_groups == 0 &&
      (c.ssm_state * c.ssm_values) % 256 == 0 && c.conv_kernel >= 1 && c.conv_kernel <= 8 &&
      c.full_interval > 0 && c.context > 0 && c.context <= (1u << 20) && c.eps > 0.0f &&
      c.rope_base > 0.0f &&
      c.kv_policy <= PRISM_B200_KV_RSQ4K3V &&
      (c.kv_policy < PRISM_B200_KV_RSQ4 || c.context <= (uint32_t)kKvqMaxPos) &&
      (c.weight_kind == PRISM_B200_KIND_TQ2_0 || c.weight_kind == PRISM_B200_KIND_Q2_K) &&
      c.hidden / 256 <= (uint32_t)kMaxNb && c.ffn / 256 <= (uint32_t)kMaxNb &&
      c.heads * c.head_dim / 256 <= (uint32_t)kMaxNb;
  if (!ok) return ex->fail(PRISM_B200_E_UNSUPPORTED, "unsupported Qwen35 geometry");
  cudaSetDevice(ex->device);
  auto *m = new prism_b200_model();
  static std::atomic<uint64_t> next_serial{1};
  m->serial = next_serial.fetch_add(1);
  m->ex = ex;
  m->cfg = c;
  m->L.resize(c.layers);
  cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  const size_t big = std::max<size_t>({c.hidden, c.ffn, (size_t)c.heads * c.head_dim * 2,
                                       (size_t)m->channels(), (size_t)m->value_width()});
#define A(p, n) \
  if (e == cudaSuccess) e = model_alloc(m, &(p), (n))
  A(m->hidden, c.hidden);
  A(m->mixed, m->channels());
  A(m->zgate, m->value_width());
  A(m->beta, c.ssm_values);
  A(m->alpha, c.ssm_values);
  A(m->attended, big);
  A(m->projected, (size_t)c.heads * c.head_dim * 2);
  A(m->key, m->kvw());
  A(m->value, m->kvw());
  A(m->up, c.ffn);
  A(m->gatef, c.ffn);
  A(m->logits, c.vocab);
  A(m->d_position, 1);
  A(m->d_tokens, (size_t)c.context + 1);
  A(m->d_prompt_end, 1);
  A(m->d_argmax, 1);
  A(m->out_norm, c.hidden);
  A(m->gdn_o, m->value_width());
  A(m->d_fsync, 4);
  A(m->d_fkey, 1);
  A(m->t_hidden, c.hidden);
  A(m->t_mixed, m->channels());
  A(m->t_z, m->value_width());
  A(m->t_beta, c.ssm_values);
  A(m->t_alpha, c.ssm_values);
  A(m->t_o, m->value_width());
  A(m->t_zs, m->value_width());
  A(m->t_proj, (size_t)c.heads * c.head_dim * 2);
  A(m->t_key, m->kvw());
  A(m->t_value, m->kvw());
  A(m->t_att, (size_t)c.heads * c.head_dim);
  A(m->t_up, c.ffn);
  A(m->t_scores, (size_t)c.heads * c.context);
  if (e == cudaSuccess) {
    // tags carry the step epoch; it starts at 1 so that no zero-filled word
    // matches, and it only grows (reset keeps it)
    const unsigned one = 1u;
    e = cudaMemcpy(m->d_fsync + 2, &one, 4, cudaMemcpyHostToDevice);
  }
  {
    const char *tr = getenv("PRISM_B200_TRACE");
    if (tr && tr[0] == '1') {
      m->nseqtrace = 5 * (int)c.layers + 1;
      A(m->d_seqtrace, (size_t)8 * m->nseqtrace);
    }
  }
  for (uint32_t l = 0; l < c.layers; ++l) {
    ModelLayer &Ly = m->L[l];
    Ly.full = m->is_full((int)l);
    A(Ly.attn_norm, c.hidden);
    A(Ly.post_norm, c.hidden);
    if (Ly.full) {
      A(Ly.q_norm, c.head_dim);
      A(Ly.k_norm, c.head_dim);
      A(Ly.kc, ((size_t)c.context * m->kv_row_bytes() + 1) / 2);
      A(Ly.vc, ((size_t)c.context * m->kv_row_bytes(true) + 1) / 2);
    } else {
      A(Ly.conv_w, (size_t)m->channels() * c.conv_kernel);
      A(Ly.dt_bias, c.ssm_values);
      A(Ly.ssm_a, c.ssm_values);
      A(Ly.ssm_norm, c.ssm_state);
      A(Ly.conv_state, (size_t)2 * m->channels() * (c.conv_kernel - 1));
      A(Ly.matrix, (size_t)c.ssm_values * c.ssm_state * c.ssm_state);
    }
  }
#undef A
  if (e != cudaSuccess) {
    prism_b200_model_destroy(m);
    return cuda_fail(ex, e, "model allocation");
  }
  *out = m;
  return PRISM_B200_OK;
}

void prism_b200_model_destroy(prism_b200_model *m) {
  if (!m) return;
  cudaSetDevice(m->ex->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  if (m->g_ingest) cudaGraphExecDestroy(m->g_ingest);
  if (m->g_decode) cudaGraphExecDestroy(m->g_decode);
  auto free_w = [](prism::DeviceWeight &w) {
    if (w.units) cudaFree(w.units);
    w.units = nullptr;
  };
  free_w(m->embd);
  for (auto &Ly : m->L) {
    for (auto *w : {&Ly.gate, &Ly.up, &Ly.down, &Ly.q, &Ly.k, &Ly.v, &Ly.o, &Ly.qkv, &Ly.z,
                    &Ly.beta, &Ly.alpha, &Ly.out})
      free_w(*w);
  }
  for (void *p : m->allocations) cudaFree(p);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

int prism_b200_model_set_tensor(prism_b200_model *m, const char *name,
                                const prism_b200_tensor *t) {
  using namespace prism;
  if (!m || !name || !t || !t->data) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  const auto &c = m->cfg;
  std::string suffix;
  const int l = parse_layer(name, suffix);
  DeviceWeight *dst = nullptr;
  uint64_t rows = 0, cols = 0;
  if (l == -1 && suffix == "token_embd.weight") {
    dst = &m->embd;
    rows = c.vocab;
    cols = c.hidden;
  } else if (l >= 0 && l < (int)c.layers) {
    ModelLayer &Ly = m->L[l];
    const uint64_t hd = c.head_dim;
    struct Slot {
      const char *n;
      DeviceWeight *w;
      uint64_t rows, cols;
      bool full;
    } slots[] = {
        {"ffn_gate.weight", &Ly.gate, c.ffn, c.hidden, Ly.full},
        {"ffn_up.weight", &Ly.up, c.ffn, c.hidden, Ly.full},
        {"ffn_down.weight", &Ly.down, c.hidden, c.ffn, Ly.full},
        {"attn_q.weight", &Ly.q, c.heads * hd * 2, c.hidden, true},
        {"attn_k.weight", &Ly.k, c.kv_heads * hd, c.hidden, true},
        {"attn_v.weight", &Ly.v, c.kv_heads * hd, c.hidden, true},
        {"attn_output.weight", &Ly.o, c.hidden, c.heads * hd, true},
        {"attn_qkv.weight", &Ly.qkv, (uint64_t)m->channels(), c.hidden, false},
        {"attn_gate.weight", &Ly.z, (uint64_t)m->value_width(), c.hidden, false},
        {"ssm_beta.weight", &Ly.beta, c.ssm_values, c.hidden, false},
        {"ssm_alpha.weight", &Ly.alpha, c.ssm_values, c.hidden, false},
        {"ssm_out.weight", &Ly.out, c.hidden, (uint64_t)m->value_width(), false},
    };
    for (auto &sl : slots)
      if (suffix == sl.n && sl.full == Ly.full) {
        dst = sl.w;
        rows = sl.rows;
        cols = sl.cols;
      }
  }
  if (!dst) return ex->fail(PRISM_B200_E_INVALID, "unknown or misplaced tensor %s", name);
  if (t->kind != c.weight_kind || t->rows != rows || t->cols != cols)
    return ex->fail(PRISM_B200_E_INVALID, "tensor %s: kind %u %llux%llu, expected %u %llux%llu",
                    name, t->kind, (unsigned long long)t->cols, (unsigned long long)t->rows,
                    c.weight_kind, (unsigned long long)cols, (unsigned long long)rows);
  const uint8_t *src = static_cast<const uint8_t *>(t->data);
  if (!scales_finite(t->kind, src, (size_t)rows * (cols / 256)))
    return ex->fail(PRISM_B200_E_NONFINITE, "tensor %s has a nonfinite block scale", name);
  cudaSetDevice(ex->device);
  if (dst->units) cudaFree(dst->units);
  dst->units = nullptr;
  cudaError_t e = upload_tiled(src, t->kind, rows, cols, ex->num_sms, m->stream, *dst);
  if (e != cudaSuccess) return cuda_fail(ex, e, "tensor upload");
  m->bound[name] = true;
  m->finalized = false;
  return PRISM_B200_OK;
}

int prism_b200_model_set_vector(prism_b200_model *m, const char *name, const float *data,
                                size_t n) {
  using namespace prism;
  if (!m || !name || !data) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  const auto &c = m->cfg;
  std::string suffix;
  const int l = parse_layer(name, suffix);
  float *dst = nullptr;
  size_t want = 0;
  if (l == -1 && suffix == "output_norm.weight") {
    dst = m->out_norm;
    want = c.hidden;
  } else if (l >= 0 && l < (int)c.layers) {
    ModelLayer &Ly = m->L[l];
    struct Slot {
      const char *n;
      float *p;
      size_t size;
    } slots[] = {
        {"attn_norm.weight", Ly.attn_norm, c.hidden},
        {"post_attention_norm.weight", Ly.post_norm, c.hidden},
        {"attn_q_norm.weight", Ly.q_norm, c.head_dim},
        {"attn_k_norm.weight", Ly.k_norm, c.head_dim},
        {"ssm_conv1d.weight", Ly.conv_w, (size_t)m->channels() * c.conv_kernel},
        {"ssm_dt.bias", Ly.dt_bias, c.ssm_values},
        {"ssm_a", Ly.ssm_a, c.ssm_values},
        {"ssm_norm.weight", Ly.ssm_norm, c.ssm_state},
    };
    for (auto &sl : slots)
      if (suffix == sl.n && sl.p) {
        dst = sl.p;
        want = sl.size;
      }
  }
  if (!dst) return ex->fail(PRISM_B200_E_INVALID, "unknown or misplaced vector %s", name);
  if (n != want) return ex->fail(PRISM_B200_E_INVALID, "vector %s has %zu values, expected %zu",
                                 name, n, want);
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(data[i]))
      return ex->fail(PRISM_B200_E_NONFINITE, "vector %s is not finite", name);
  if (suffix == "ssm_a")
    for (size_t i = 0; i < n; ++i)
      if (data[i] > 0.0f)
        return ex->fail(PRISM_B200_E_INVALID, "recurrent decay ssm_a must be nonpositive");
  cudaSetDevice(ex->device);
  cudaError_t e = cudaMemcpy(dst, data, n * sizeof(float), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(ex, e, "vector upload");
  m->bound[name] = true;
  return PRISM_B200_OK;
}

int prism_b200_model_finalize(prism_b200_model *m) {
  using namespace prism;
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  std::vector<std::string> need = {"token_embd.weight", "output_norm.weight"};
  for (uint32_t l = 0; l < m->cfg.layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    for (const char *s : {"attn_norm.weight", "post_attention_norm.weight", "ffn_gate.weight",
                          "ffn_up.weight", "ffn_down.weight"})
      need.push_back(p + s);
    if (m->L[l].full) {
      for (const char *s : {"attn_q.weight", "attn_k.weight", "attn_v.weight",
                            "attn_output.weight", "attn_q_norm.weight", "attn_k_norm.weight"})
        need.push_back(p + s);
    } else {
      for (const char *s : {"attn_qkv.weight", "attn_gate.weight", "ssm_beta.weight",
                            "ssm_alpha.weight", "ssm_out.weight", "ssm_conv1d.weight",
                            "ssm_dt.bias", "ssm_a", "ssm_norm.weight"})
        need.push_back(p + s);
    }
  }
  for (auto &n : need)
    if (!m->bound.count(n)) return ex->fail(PRISM_B200_E_INVALID, "tensor %s is not bound", n.c_str());
  cudaSetDevice(ex->device);
  if (m->g_ingest) cudaGraphExecDestroy(m->g_ingest);
  if (m->g_decode) cudaGraphExecDestroy(m->g_decode);
  m->g_ingest = m->g_decode = nullptr;
  cudaError_t e = prepare_flow(m);
  if (e != cudaSuccess) return cuda_fail(ex, e, "dataflow step setup");
  e = capture_step(m, false, &m->g_ingest);
  if (e == cudaSuccess) e = capture_step(m, true, &m->g_decode);
  if (e != cudaSuccess) return cuda_fail(ex, e, "step graph capture");
  m->finalized = true;
  return prism_b200_model_reset(m);
}

int prism_b200_model_reset(prism_b200_model *m) {
  using namespace prism;
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  cudaSetDevice(ex->device);
  const auto &c = m->cfg;
  cudaStream_t s = m->stream;
  for (auto &Ly : m->L) {
    if (Ly.full) {
      CK(cudaMemsetAsync(Ly.kc, 0, (size_t)c.context * m->kv_row_bytes(), s), "reset");
      CK(cudaMemsetAsync(Ly.vc, 0, (size_t)c.context * m->kv_row_bytes(true), s), "reset");
    } else {
      CK(cudaMemsetAsync(Ly.conv_state, 0, (size_t)2 * m->channels() * (c.conv_kernel - 1) * 4, s),
         "reset");
      CK(cudaMemsetAsync(Ly.matrix, 0, (size_t)c.ssm_values * c.ssm_state * c.ssm_state * 4, s),
         "reset");
    }
  }
  CK(cudaMemsetAsync(m->d_fsync, 0, 2 * 4, s), "reset");
  CK(cudaMemsetAsync(m->d_fkey, 0, 8, s), "reset");
  CK(cudaMemsetAsync(m->d_position, 0, 4, s), "reset");
  CK(cudaMemsetAsync(m->d_tokens, 0, ((size_t)c.context + 1) * 4, s), "reset");
  CK(cudaStreamSynchronize(s), "reset");
  m->position = 0;
  return PRISM_B200_OK;
}

int64_t prism_b200_model_position(const prism_b200_model *m) { return m ? m->position : -1; }

int prism_b200_model_persistent(const prism_b200_model *m) { return m && m->flow ? 1 : 0; }

int64_t prism_b200_model_phase_trace_ctas(prism_b200_model *m, uint64_t *ns, size_t count) {
  if (!m || !ns) return -PRISM_B200_E_INVALID;
  if (!m->flow) return 0;
  const size_t n = std::min(count, (size_t)4 * m->ex->num_sms * m->nfphases);
  if (cudaMemcpy(ns, m->d_ftrace_cta, n * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
    return -PRISM_B200_E_DEVICE;
  return (int64_t)n;
}

int prism_b200_model_step_mode(const prism_b200_model *m) {
  return !m ? -1 : m->flow ? 2 : 0;
}

int64_t prism_b200_model_phase_trace(prism_b200_model *m, uint64_t *ns, size_t count) {
  if (!m || !ns) return -PRISM_B200_E_INVALID;
  if (m->flow) {
    const size_t n = std::min(count, (size_t)16 * m->nfphases);
    if (cudaMemcpy(ns, m->d_ftrace, n * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
      return -PRISM_B200_E_DEVICE;
    return (int64_t)n;
  }
  // the kernel-sequence step's per-launch timelines, when enabled
  if (!m->d_seqtrace) return 0;
  const size_t n = std::min(count, (size_t)8 * m->nseqtrace);
  if (cudaMemcpy(ns, m->d_seqtrace, n * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
    return -PRISM_B200_E_DEVICE;
  return (int64_t)n;
}

static int model_finish(prism_b200_model *m) {
  prism_b200_executor *ex = m->ex;
  CK(cudaMemcpyAsync(ex->h_status, ex->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost,
                     m->stream),
     "status readback");
  CK(cudaStreamSynchronize(m->stream), "model step");
  if (*ex->h_status) {
    ex->faulted = true;
    return ex->fail(status_to_code(*ex->h_status), "device reported status 0x%x",
                    *ex->h_status);
  }
  return PRISM_B200_OK;
}

int prism_b200_model_evaluate(prism_b200_model *m, uint32_t token, float *logits,
                              uint32_t *greedy) {
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (token >= m->cfg.vocab || m->position >= (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID,
                    "token is outside the vocabulary or context is exhausted");
  cudaSetDevice(ex->device);
  cudaStream_t s = m->stream;
  const int never = 0x7fffffff;
  CK(cudaMemcpyAsync(m->d_tokens + m->position, &token, 4, cudaMemcpyHostToDevice, s), "token");
  CK(cudaMemcpyAsync(m->d_prompt_end, &never, 4, cudaMemcpyHostToDevice, s), "token");
  CK(cudaGraphLaunch(m->g_decode, s), "decode step");
  unsigned long long key = 0;
  CK(cudaMemcpyAsync(&key, m->d_argmax, 8, cudaMemcpyDeviceToHost, s), "greedy");
  if (logits)
    CK(cudaMemcpyAsync(logits, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s),
       "logits");
  st = model_finish(m);
  if (st) {
    if (logits) memset(logits, 0, (size_t)m->cfg.vocab * 4);
    return st;
  }
  m->position += 1;
  if (greedy) *greedy = 0xffffffffu - (uint32_t)(key & 0xffffffffull);
  return PRISM_B200_OK;
}

int prism_b200_model_decode_async(prism_b200_model *m, size_t steps) {
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (m->position + (int64_t)steps > (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  cudaSetDevice(ex->device);
  for (size_t i = 0; i < steps; ++i) CK(cudaGraphLaunch(m->g_decode, m->stream), "decode step");
  m->position += (int64_t)steps;
  return PRISM_B200_OK;
}

void *prism_b200_model_stream(const prism_b200_model *m) {
  return m ? reinterpret_cast<void *>(m->stream) : nullptr;
}

int prism_b200_model_set_prompt(prism_b200_model *m, const uint32_t *tokens, size_t n) {
  if (!m || !tokens || n == 0) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  if (m->position + (int64_t)n > (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= m->cfg.vocab)
      return ex->fail(PRISM_B200_E_INVALID, "prompt token outside the vocabulary");
  cudaSetDevice(ex->device);
  const int end = (int)(m->position + (int64_t)n);
  CK(cudaMemcpyAsync(m->d_tokens + m->position, tokens, n * 4, cudaMemcpyHostToDevice, m->stream),
     "prompt");
  CK(cudaMemcpyAsync(m->d_prompt_end, &end, 4, cudaMemcpyHostToDevice, m->stream), "prompt");
  CK(cudaStreamSynchronize(m->stream), "prompt");
  return PRISM_B200_OK;
}

int prism_b200_model_ingest_async(prism_b200_model *m, size_t n) {
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (m->position + (int64_t)n > (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  cudaSetDevice(ex->device);
  for (size_t i = 0; i < n; ++i) CK(cudaGraphLaunch(m->g_ingest, m->stream), "ingest step");
  m->position += (int64_t)n;
  return PRISM_B200_OK;
}

int prism_b200_model_generate(prism_b200_model *m, const uint32_t *prompt, size_t n_prompt,
                              size_t n_new, uint32_t *out) {
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (!prompt || n_prompt == 0 || (n_new && !out))
    return ex->fail(PRISM_B200_E_INVALID, "generation needs a prompt");
  if (m->position + (int64_t)n_prompt + (int64_t)n_new > (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  for (size_t i = 0; i < n_prompt; ++i)
    if (prompt[i] >= m->cfg.vocab)
      return ex->fail(PRISM_B200_E_INVALID, "prompt token outside the vocabulary");
  cudaSetDevice(ex->device);
  cudaStream_t s = m->stream;
  const int end = (int)(m->position + (int64_t)n_prompt);
  CK(cudaMemcpyAsync(m->d_tokens + m->position, prompt, n_prompt * 4, cudaMemcpyHostToDevice, s),
     "prompt");
  CK(cudaMemcpyAsync(m->d_prompt_end, &end, 4, cudaMemcpyHostToDevice, s), "prompt");
  for (size_t i = 0; i + 1 < n_prompt; ++i) CK(cudaGraphLaunch(m->g_ingest, s), "ingest step");
  const size_t decode_steps = n_new ? n_new : 1;
  for (size_t i = 0; i < decode_steps; ++i) CK(cudaGraphLaunch(m->g_decode, s), "decode step");
  if (n_new)
    CK(cudaMemcpyAsync(out, m->d_tokens + end, n_new * 4, cudaMemcpyDeviceToHost, s), "tokens");
  st = model_finish(m);
  if (st) return st;
  m->position += (int64_t)(n_prompt - 1 + decode_steps);
  return PRISM_B200_OK;
}

int prism_b200_model_step_timings(prism_b200_model *m, float *attention_ms, float *ffn_ms,
                                  float *head_ms, float *total_ms) {
  if (!m) return PRISM_B200_E_INVALID;
  prism_b200_executor *ex = m->ex;
  int st = check_open(ex);
  if (st) return st;
  if (!m->finalized) return ex->fail(PRISM_B200_E_INVALID, "model is not finalized");
  if (m->position >= (int64_t)m->cfg.context)
    return ex->fail(PRISM_B200_E_INVALID, "context is exhausted");
  cudaSetDevice(ex->device);
  const int nl = (int)m->L.size();
  if (m->flow) {
    // one traced dataflow step: CTA 0's phase ends (each phase's input wait
    // counted in the phase)
    std::vector<unsigned long long> t((size_t)16 * m->nfphases);
    cudaError_t e = cudaMemsetAsync(m->d_ftrace, 0, t.size() * 8, m->stream);
    if (e == cudaSuccess) e = prism::launch_flow(m, true, true);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess)
      e = cudaMemcpy(t.data(), m->d_ftrace, t.size() * 8, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(ex, e, "traced step");
    auto end = [&](int q) { return t[(size_t)16 * q + 7]; };
    auto ms = [](unsigned long long a, unsigned long long b) {
      return (float)((double)(b - a) * 1e-6);
    };
    int p = 1;  // phase 0 is the embedding
    for (int l = 0; l < nl; ++l) {
      const int ffn = p + 3;  // three attention-side phases, then the FFN pair
      if (attention_ms) attention_ms[l] = ms(end(p - 1), end(ffn - 1));
      if (ffn_ms) ffn_ms[l] = ms(end(ffn - 1), end(ffn + 1));
      p = ffn + 2;
    }
    if (head_ms) *head_ms = ms(end(p - 1), end(p));
    if (total_ms) *total_ms = ms(t[0], end(m->nfphases - 1));
    st = model_finish(m);
    if (st) return st;
    m->position += 1;
    return PRISM_B200_OK;
  }
  std::vector<cudaEvent_t> ev((size_t)(2 * nl + 4));
  for (auto &e : ev) CK(cudaEventCreate(&e), "event");
  cudaError_t e = prism::enqueue_step(m, true, ev.data());
  if (e == cudaSuccess) e = cudaEventSynchronize(ev.back());
  if (e == cudaSuccess) {
    auto span = [&](int a, int b) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, ev[a], ev[b]);
      return ms;
    };
    for (int l = 0; l < nl; ++l) {
      if (attention_ms) attention_ms[l] = span(1 + 2 * l, 2 + 2 * l);
      if (ffn_ms) ffn_ms[l] = span(2 + 2 * l, 3 + 2 * l);
    }
    if (head_ms) *head_ms = span(1 + 2 * nl, 2 + 2 * nl);
    if (total_ms) *total_ms = span(0, 3 + 2 * nl);
  }
  for (auto &x : ev) cudaEventDestroy(x);
  if (e != cudaSuccess) return cuda_fail(ex, e, "timed step");
  st = model_finish(m);
  if (st) return st;
  m->position += 1;
  return PRISM_B200_OK;
}

int64_t prism_b200_model_read_state(prism_b200_model *m, uint32_t layer, uint32_t which,
                                    void *out, size_t bytes) {
  if (!m || !out) return -PRISM_B200_E_INVALID;
  const auto &c = m->cfg;
  const void *src = nullptr;
  size_t n = 0;
  if (which == 4) {
    src = m->hidden;
    n = (size_t)c.hidden * 4;
  } else if (which >= 5 && which <= 9) {
    // the last layer's activations: 5 attended, 6 gate projection (GDN),
    // 7 ffn up projection, 8 ffn gate projection, 9 logits
    const size_t sizes[5] = {(size_t)std::max(m->value_width(), (int)(c.heads * c.head_dim)),
                             (size_t)m->value_width(), c.ffn, c.ffn, c.vocab};
    const void *ptrs[5] = {m->attended, m->zgate, m->up, m->gatef, m->logits};
    src = ptrs[which - 5];
    n = sizes[which - 5] * 4;
  } else if (layer < c.layers) {
    const prism::ModelLayer &Ly = m->L[layer];
    const size_t hist = (size_t)m->channels() * (c.conv_kernel - 1);
    if (which == 0 && !Ly.full) {
      // the buffer written by the last step: parity of the current position
      src = Ly.conv_state + (m->position & 1) * hist;
      n = hist * 4;
    } else if (which == 1 && !Ly.full) {
      src = Ly.matrix;
      n = (size_t)c.ssm_values * c.ssm_state * c.ssm_state * 4;
    } else if ((which == 2 || which == 3) && Ly.full) {
      src = which == 2 ? Ly.kc : Ly.vc;
      n = (size_t)m->position * m->kv_row_bytes(which == 3);
    }
  }
  if (!src) return -PRISM_B200_E_INVALID;
  if (bytes < n) return -PRISM_B200_E_INVALID;
  cudaSetDevice(m->ex->device);
  if (cudaMemcpyAsync(out, src, n, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess ||
      cudaStreamSynchronize(m->stream) != cudaSuccess)
    return -PRISM_B200_E_DEVICE;
  return (int64_t)n;
}

}  // extern "C"
