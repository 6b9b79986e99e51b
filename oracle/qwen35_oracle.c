/*
 * qwen35_oracle.c -- CPU restatement of the reference's Qwen35 decode step
 * (Source arithmetic).  TEST INFRASTRUCTURE ONLY: the parity checker and
 * CPU baseline for the B200 model path; never part of the product library.
 *
 * Layer order follows reference src/graph.rs:3789-4033
 * (evaluate_hidden_with_executor): RMSNorm -> attention (full or GDN) ->
 * residual add + RMSNorm -> up/gate -> SwiGLU -> down -> residual add; after
 * the last layer: RMSNorm -> tied output projection.
 */
#include "qwen35_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "prism_oracle.h"

struct po_qwen35 {
  po_qwen35_config cfg;
  const uint8_t *embd;
  const float *out_norm;
  const void **w; /* layers * PO_W_PER_LAYER */
  int32_t position;
  float **conv;       /* per layer: [channels][k-1] (recurrent only) */
  float **matrix;     /* per layer: [values][S][S] */
  uint16_t **keys;    /* per layer: [context][kv*hd] (full only) */
  uint16_t **vals;
  /* scratch */
  float *hidden, *normalized, *attn_out, *mixed, *zgate, *beta, *alpha, *attended;
  float *projected, *key, *value, *query, *scores, *up, *gate, *down, *next_matrix,
      *next_conv, *freqs;
  po_q8k_block *act;
};

static inline int key_width(const po_qwen35_config *c) { return c->ssm_state * c->ssm_groups; }
static inline int value_width(const po_qwen35_config *c) { return c->ssm_state * c->ssm_values; }
static inline int conv_channels(const po_qwen35_config *c) {
  return 2 * key_width(c) + value_width(c);
}
static inline int block_bytes_of(const po_qwen35_config *c) { return po_block_bytes(c->weight_kind); }

int po_qwen35_is_full_layer(const po_qwen35_config *cfg, int layer) {
  return ((layer + 1) % cfg->full_interval) == 0;
}

static const void *W(const po_qwen35 *m, int layer, int slot) {
  return m->w[(size_t)layer * PO_W_PER_LAYER + slot];
}

#define ALLOC(p, n) ((p) = calloc((size_t)(n), sizeof(*(p))))

po_qwen35 *po_qwen35_create(const po_qwen35_config *cfg, const void *const *globals,
                            const void *const *layers) {
  po_qwen35 *m = calloc(1, sizeof(po_qwen35));
  if (!m) return NULL;
  m->cfg = *cfg;
  m->embd = (const uint8_t *)globals[0];
  m->out_norm = (const float *)globals[1];
  size_t nw = (size_t)cfg->layers * PO_W_PER_LAYER;
  ALLOC(m->w, nw);
  memcpy(m->w, layers, nw * sizeof(void *));
  ALLOC(m->conv, cfg->layers);
  ALLOC(m->matrix, cfg->layers);
  ALLOC(m->keys, cfg->layers);
  ALLOC(m->vals, cfg->layers);
  const int S = cfg->ssm_state, kvw = cfg->kv_heads * cfg->head_dim;
  for (int l = 0; l < cfg->layers; ++l) {
    if (po_qwen35_is_full_layer(cfg, l)) {
      ALLOC(m->keys[l], (size_t)cfg->context * kvw);
      ALLOC(m->vals[l], (size_t)cfg->context * kvw);
    } else {
      ALLOC(m->conv[l], (size_t)conv_channels(cfg) * (cfg->conv_kernel - 1));
      ALLOC(m->matrix[l], (size_t)cfg->ssm_values * S * S);
    }
  }
  int big = cfg->hidden;
  int cand[] = {cfg->ffn, cfg->heads * cfg->head_dim * 2, conv_channels(cfg), value_width(cfg)};
  for (int i = 0; i < 4; ++i)
    if (cand[i] > big) big = cand[i];
  ALLOC(m->hidden, cfg->hidden);
  ALLOC(m->normalized, cfg->hidden);
  ALLOC(m->attn_out, cfg->hidden);
  ALLOC(m->mixed, conv_channels(cfg));
  ALLOC(m->zgate, value_width(cfg));
  ALLOC(m->beta, cfg->ssm_values);
  ALLOC(m->alpha, cfg->ssm_values);
  ALLOC(m->attended, big);
  ALLOC(m->projected, cfg->heads * cfg->head_dim * 2);
  ALLOC(m->key, kvw);
  ALLOC(m->value, kvw);
  ALLOC(m->query, cfg->heads * cfg->head_dim);
  ALLOC(m->scores, cfg->context + 1);
  ALLOC(m->up, cfg->ffn);
  ALLOC(m->gate, cfg->ffn);
  ALLOC(m->down, cfg->hidden);
  ALLOC(m->next_matrix, (size_t)cfg->ssm_values * S * S);
  ALLOC(m->next_conv, (size_t)conv_channels(cfg) * (cfg->conv_kernel - 1));
  ALLOC(m->freqs, cfg->rope_dim);
  ALLOC(m->act, big / 256 + 1);
  return m;
}

void po_qwen35_destroy(po_qwen35 *m) {
  if (!m) return;
  for (int l = 0; l < m->cfg.layers; ++l) {
    free(m->conv[l]);
    free(m->matrix[l]);
    free(m->keys[l]);
    free(m->vals[l]);
  }
  free(m->conv); free(m->matrix); free(m->keys); free(m->vals); free(m->w);
  free(m->hidden); free(m->normalized); free(m->attn_out); free(m->mixed); free(m->zgate);
  free(m->beta); free(m->alpha); free(m->attended); free(m->projected); free(m->key);
  free(m->value); free(m->query); free(m->scores); free(m->up); free(m->gate); free(m->down);
  free(m->next_matrix); free(m->next_conv); free(m->freqs); free(m->act);
  free(m);
}

void po_qwen35_reset(po_qwen35 *m) {
  const po_qwen35_config *c = &m->cfg;
  const int S = c->ssm_state, kvw = c->kv_heads * c->head_dim;
  for (int l = 0; l < c->layers; ++l) {
    if (po_qwen35_is_full_layer(c, l)) {
      memset(m->keys[l], 0, (size_t)c->context * kvw * 2);
      memset(m->vals[l], 0, (size_t)c->context * kvw * 2);
    } else {
      memset(m->conv[l], 0, (size_t)conv_channels(c) * (c->conv_kernel - 1) * 4);
      memset(m->matrix[l], 0, (size_t)c->ssm_values * S * S * 4);
    }
  }
  m->position = 0;
}

int32_t po_qwen35_position(const po_qwen35 *m) { return m->position; }
const float *po_qwen35_conv_state(const po_qwen35 *m, int l) { return m->conv[l]; }
const float *po_qwen35_matrix_state(const po_qwen35 *m, int l) { return m->matrix[l]; }
const uint16_t *po_qwen35_keys(const po_qwen35 *m, int l) { return m->keys[l]; }
const uint16_t *po_qwen35_values(const po_qwen35 *m, int l) { return m->vals[l]; }
const float *po_qwen35_hidden(const po_qwen35 *m) { return m->hidden; }

int po_qwen35_load_state(po_qwen35 *m, int layer, int which, const void *src, size_t bytes) {
  const po_qwen35_config *c = &m->cfg;
  if (layer < 0 || layer >= c->layers || !src) return PO_E_INVALID;
  const int full = po_qwen35_is_full_layer(c, layer);
  void *dst = NULL;
  size_t cap = 0;
  if (which == 0 && !full) {
    dst = m->conv[layer];
    cap = (size_t)conv_channels(c) * (c->conv_kernel - 1) * 4;
  } else if (which == 1 && !full) {
    dst = m->matrix[layer];
    cap = (size_t)c->ssm_values * c->ssm_state * c->ssm_state * 4;
  } else if ((which == 2 || which == 3) && full) {
    dst = which == 2 ? (void *)m->keys[layer] : (void *)m->vals[layer];
    cap = (size_t)c->context * c->kv_heads * c->head_dim * 2;
  }
  if (!dst || bytes > cap) return PO_E_INVALID;
  memcpy(dst, src, bytes);
  return PO_OK;
}

int po_qwen35_set_position(po_qwen35 *m, int32_t position) {
  if (position < 0 || position >= m->cfg.context) return PO_E_INVALID;
  m->position = position;
  return PO_OK;
}

/* Q8_K-quantize x once, then project each weight (sibling group). */
static int project_group(po_qwen35 *m, const float *x, int cols, int n, const void *const *ws,
                         const int *rows, float *const *outs, int threads) {
  int st = po_q8k_quantize(x, (size_t)cols, 0, m->act);
  if (st) return st;
  for (int i = 0; i < n; ++i) {
    st = po_matvec(m->cfg.weight_kind, (const uint8_t *)ws[i], (size_t)rows[i], (size_t)cols,
                   m->act, outs[i], threads);
    if (st) return st;
  }
  return PO_OK;
}

/* reference src/graph.rs:6406-6437 rope_frequencies_mrope at text position p
 * (positions [p, p, p, 0]); cos_sin holds rope_dim/2 (cos, sin) pairs. */
void po_rope_frequencies(const po_qwen35_config *cfg, int position, float *cos_sin) {
  float theta_scale = powf(cfg->rope_base, -2.0f / (float)cfg->rope_dim);
  float thetas[4] = {(float)position, (float)position, (float)position, 0.0f};
  for (int i = 0; i < cfg->rope_dim / 2; ++i) {
    int sector = i % 3;
    float angle = i < 3 * cfg->rope_sections[sector] ? thetas[sector] : thetas[3];
    cos_sin[2 * i] = po_cosf(angle);
    cos_sin[2 * i + 1] = po_sinf(angle);
    for (int t = 0; t < 4; ++t) thetas[t] = thetas[t] * theta_scale;
  }
}

/* reference src/kernels.rs:3679-3750 rms_norm_rope_round_f16_into (Source) */
static int norm_rope_round(const po_qwen35_config *c, const float *in, const float *w,
                           const float *freqs, float *out) {
  int st = po_rms_norm(in, w, (size_t)c->head_dim, c->eps, out);
  if (st) return st;
  const int half = c->rope_dim / 2;
  for (int i = 0; i < half; ++i) {
    float cs = freqs[2 * i], sn = freqs[2 * i + 1];
    float first = out[i], second = out[i + half];
    out[i] = first * cs - second * sn;
    out[i + half] = first * sn + second * cs;
  }
  for (int i = 0; i < c->head_dim; ++i) {
    if (!isfinite(out[i])) return PO_E_NONFINITE;
    out[i] = po_round_f16(out[i]);
  }
  return PO_OK;
}

/* Q8_0 record of one KV head's row: scales then codes. */
static int q8_record(const float *x, int hd, uint8_t *rec) {
  po_q8_0_block blk[32];
  int st = po_q8_0_quantize(x, (size_t)hd, blk);
  if (st) return st;
  for (int j = 0; j < hd / 32; ++j) {
    memcpy(rec + 2 * j, &blk[j].d, 2);
    memcpy(rec + hd / 32 * 2 + 32 * j, blk[j].values, 32);
  }
  return PO_OK;
}

static void q8_dequant(const uint8_t *rec, int hd, float *out) {
  for (int i = 0; i < hd; ++i) {
    uint16_t d;
    memcpy(&d, rec + 2 * (i / 32), 2);
    out[i] = po_half_to_float(d) * (float)(int8_t)rec[hd / 32 * 2 + i];
  }
}

/* The attention of full_attention below over Q8_0 KV records (kv_policy 1):
 * scores are float_dot(q, dequantized key), values binary64 sums of
 * binary32 products with the dequantized values; the current position is
 * quantized first and read back like the history. */
static int q8_attention(po_qwen35 *m, int l, float scale, int threads) {
  const po_qwen35_config *c = &m->cfg;
  const int hd = c->head_dim, rb = PO_KV_Q8_0_RECORD(hd);
  const int npos = m->position, group = c->heads / c->kv_heads;
  uint8_t *krec = (uint8_t *)m->keys[l], *vrec = (uint8_t *)m->vals[l];
  const size_t pstride = (size_t)c->kv_heads * rb;
  int st;
  for (int k = 0; k < c->kv_heads; ++k) {
    if ((st = q8_record(m->key + (size_t)k * hd, hd, krec + npos * pstride + (size_t)k * rb)))
      return st;
    if ((st = q8_record(m->value + (size_t)k * hd, hd, vrec + npos * pstride + (size_t)k * rb)))
      return st;
  }
  float kd[1024], vd[1024];
  for (int h = 0; h < c->heads; ++h) {
    const int kh = h / group;
    const float *q = m->query + (size_t)h * hd;
    for (int p = 0; p <= npos; ++p) {
      q8_dequant(krec + p * pstride + (size_t)kh * rb, hd, kd);
      m->scores[p] = po_float_dot(q, kd, (size_t)hd) * scale;
    }
    if ((st = po_softmax_round_f16(m->scores, (size_t)npos + 1))) return st;
    const float *g = m->projected + (size_t)(2 * h + 1) * hd;
    float *out = m->attended + (size_t)h * hd;
    double sums[1024];
    for (int d = 0; d < hd; ++d) sums[d] = -0.0;
    for (int p = 0; p < npos; ++p) {
      q8_dequant(vrec + p * pstride + (size_t)kh * rb, hd, vd);
      for (int d = 0; d < hd; ++d) sums[d] += (double)(m->scores[p] * vd[d]);
    }
    q8_dequant(vrec + npos * pstride + (size_t)kh * rb, hd, vd);
    for (int d = 0; d < hd; ++d) {
      float v = (float)(sums[d] + (double)(m->scores[npos] * vd[d]));
      out[d] = v * (1.0f / (1.0f + po_expf(-g[d])));
    }
  }
  const void *wo[1] = {W(m, l, PO_W_O)};
  int ro[1] = {c->hidden};
  float *oo[1] = {m->attn_out};
  return project_group(m, m->attended, c->heads * hd, 1, wo, ro, oo, threads);
}

/* The attention of full_attention below over rotated scalar KV records
 * (kv_policy 2 rsq4, 3 rsq4vf, 4 rsq4k3v; reference src/graph/
 * quantized_kv.rs:16-84 KvCachePolicy and :629-657 prepare_current): the
 * current position's normalised key and rounded value are encoded first
 * (key: 4 bits, the key seed; value: 4 or 3 bits, the value seed, version 2
 * for rsq4vf) and every position, the current one included, is read back as
 * a record by attend_head. */
#define KVQ_KEY_SEED 0x53574946544b5631ull
#define KVQ_VALUE_SEED 0x5357494654565631ull
static int kvq_attention(po_qwen35 *m, int l, float scale) {
  const po_qwen35_config *c = &m->cfg;
  const int hd = c->head_dim, npos = m->position, group = c->heads / c->kv_heads;
  const int vbits = c->kv_policy == 4 ? 3 : 4, vversion = c->kv_policy == 3 ? 2 : 1;
  const int kb = po_kvq_record_bytes(4), vb = po_kvq_record_bytes(vbits);
  uint8_t *krec = (uint8_t *)m->keys[l], *vrec = (uint8_t *)m->vals[l];
  int st;
  for (int k = 0; k < c->kv_heads; ++k) {
    if ((st = po_kvq_encode(4, KVQ_KEY_SEED, 1, m->key + (size_t)k * hd,
                            krec + ((size_t)npos * c->kv_heads + k) * kb)))
      return st;
    if ((st = po_kvq_encode(vbits, KVQ_VALUE_SEED, vversion, m->value + (size_t)k * hd,
                            vrec + ((size_t)npos * c->kv_heads + k) * vb)))
      return st;
  }
  /* attend_head takes one KV head's records contiguous: gather them */
  uint8_t *kk = (uint8_t *)malloc((size_t)(npos + 1) * kb);
  uint8_t *vv = (uint8_t *)malloc((size_t)(npos + 1) * vb);
  if (!kk || !vv) {
    free(kk);
    free(vv);
    return PO_E_INVALID;
  }
  st = PO_OK;
  for (int h = 0; h < c->heads && !st; ++h) {
    const int kh = h / group;
    if (h % group == 0)
      for (int p = 0; p <= npos; ++p) {
        memcpy(kk + (size_t)p * kb, krec + ((size_t)p * c->kv_heads + kh) * kb, (size_t)kb);
        memcpy(vv + (size_t)p * vb, vrec + ((size_t)p * c->kv_heads + kh) * vb, (size_t)vb);
      }
    st = po_kvq_attend_head(4, KVQ_KEY_SEED, vbits, KVQ_VALUE_SEED, m->query + (size_t)h * hd, kk,
                            vv, (size_t)npos + 1, scale, m->projected + (size_t)(2 * h + 1) * hd,
                            m->attended + (size_t)h * hd);
  }
  free(kk);
  free(vv);
  return st;
}

/* reference src/graph.rs:4383-4950 full_attention (F16 KV, Source) */
static int full_attention(po_qwen35 *m, int l, int threads) {
  const po_qwen35_config *c = &m->cfg;
  const int hd = c->head_dim, kvw = c->kv_heads * hd;
  const void *ws[3] = {W(m, l, PO_W_Q), W(m, l, PO_W_K), W(m, l, PO_W_V)};
  int rows[3] = {c->heads * hd * 2, kvw, kvw};
  float *outs[3] = {m->projected, m->key, m->value};
  int st = project_group(m, m->normalized, c->hidden, 3, ws, rows, outs, threads);
  if (st) return st;
  po_rope_frequencies(c, m->position, m->freqs);
  const float *qn = (const float *)W(m, l, PO_W_Q_NORM);
  const float *kn = (const float *)W(m, l, PO_W_K_NORM);
  for (int h = 0; h < c->heads; ++h)
    if ((st = norm_rope_round(c, m->projected + (size_t)h * 2 * hd, qn, m->freqs,
                              m->query + (size_t)h * hd)))
      return st;
  float tmp[1024];
  for (int k = 0; k < c->kv_heads; ++k) {
    if ((st = norm_rope_round(c, m->key + (size_t)k * hd, kn, m->freqs, tmp))) return st;
    memcpy(m->key + (size_t)k * hd, tmp, (size_t)hd * 4);
  }
  for (int i = 0; i < kvw; ++i) m->value[i] = po_round_f16(m->value[i]);
  const float scale = 1.0f / sqrtf((float)hd);
  const int npos = m->position;
  const int group = c->heads / c->kv_heads;
  if (c->kv_policy == 1) return q8_attention(m, l, scale, threads);
  if (c->kv_policy >= 2) {
    if ((st = kvq_attention(m, l, scale))) return st;
    const void *wo[1] = {W(m, l, PO_W_O)};
    int ro[1] = {c->hidden};
    float *oo[1] = {m->attn_out};
    return project_group(m, m->attended, c->heads * hd, 1, wo, ro, oo, threads);
  }
  for (int h = 0; h < c->heads; ++h) {
    const int off = (h / group) * hd;
    const float *q = m->query + (size_t)h * hd;
    for (int p = 0; p < npos; ++p)
      m->scores[p] = po_f16_dot(q, m->keys[l] + (size_t)p * kvw + off, (size_t)hd) * scale;
    m->scores[npos] = po_float_dot(q, m->key + off, (size_t)hd) * scale;
    if ((st = po_softmax_round_f16(m->scores, (size_t)npos + 1))) return st;
    const float *g = m->projected + (size_t)(2 * h + 1) * hd;
    float *out = m->attended + (size_t)h * hd;
    for (int d = 0; d < hd; ++d) {
      double sum = -0.0;
      for (int p = 0; p < npos; ++p)
        sum += (double)(m->scores[p] * po_half_to_float(m->vals[l][(size_t)p * kvw + off + d]));
      float v = (float)(sum + (double)(m->scores[npos] * m->value[off + d]));
      out[d] = v * (1.0f / (1.0f + po_expf(-g[d])));
    }
  }
  const void *wo[1] = {W(m, l, PO_W_O)};
  int ro[1] = {c->hidden};
  float *oo[1] = {m->attn_out};
  if ((st = project_group(m, m->attended, c->heads * hd, 1, wo, ro, oo, threads))) return st;
  for (int i = 0; i < kvw; ++i) {
    m->keys[l][(size_t)npos * kvw + i] = po_float_to_half(m->key[i]);
    m->vals[l][(size_t)npos * kvw + i] = po_float_to_half(m->value[i]);
  }
  return PO_OK;
}

/* reference src/graph.rs:801-822 gdn_step_row_from (Source) per row, and
 * src/graph.rs:5191-5343 for the head loop. */
int po_gdn_head_step(const float *prev, float *next, const float *q, const float *k,
                     const float *v, float decay, float beta, int rows, int width,
                     float *out) {
  const float scale = 1.0f / sqrtf((float)width);
  for (int r = 0; r < rows; ++r) {
    const float *p = prev + (size_t)r * width;
    float *s = next + (size_t)r * width;
    for (int i = 0; i < width; ++i) s[i] = decay * p[i];
    float dk = po_float_dot(s, k, (size_t)width);
    float delta = (v[r] - dk) * beta;
    for (int i = 0; i < width; ++i) {
      s[i] = s[i] + delta * k[i];
      if (!isfinite(s[i])) return PO_E_NONFINITE;
    }
    out[r] = po_float_dot(s, q, (size_t)width) * scale;
  }
  return PO_OK;
}

/* reference src/graph/prefill_gdn.rs:143-216 exact_head_into: the decode
 * recurrence applied token after token. */
int po_gdn_head_prefill_exact(float *state, const float *q, const float *k, const float *v,
                              const float *decay, const float *beta, int T, int rows,
                              int width, float *out) {
  float *next = malloc((size_t)rows * width * sizeof(float));
  if (!next) return PO_E_INVALID;
  for (int t = 0; t < T; ++t) {
    int st = po_gdn_head_step(state, next, q + (size_t)t * width, k + (size_t)t * width,
                              v + (size_t)t * rows, decay[t], beta[t], rows, width,
                              out + (size_t)t * rows);
    if (st) {
      free(next);
      return st;
    }
    memcpy(state, next, (size_t)rows * width * sizeof(float));
  }
  free(next);
  return PO_OK;
}

/* reference src/graph/prefill_gdn.rs:223-456 head_into (chunkwise WY form,
 * separately rounded binary32 arithmetic), for chunks of up to 64 tokens.
 * For each chunk: products[t][j] = prod of decays over (j, t]; cross_key /
 * cross_query hold decayed key-key / key-query dots; per state row the
 * deltas are a forward substitution; the state is updated once per chunk. */
int po_gdn_head_prefill_chunked(float *state, const float *q, const float *k, const float *v,
                                const float *decay, const float *beta, int T, int rows,
                                int width, int chunk, float *out) {
  enum { MAXC = 64 };
  if (chunk < 1 || chunk > MAXC) return PO_E_INVALID;
  static __thread float products[MAXC][MAXC], cross_key[MAXC][MAXC], cross_query[MAXC][MAXC];
  float cumulative[MAXC], deltas[MAXC];
  float *prev = malloc((size_t)rows * width * sizeof(float));
  if (!prev) return PO_E_INVALID;
  const float scale = 1.0f / sqrtf((float)width);
  for (int c0 = 0; c0 < T; c0 += chunk) {
    const int count = T - c0 < chunk ? T - c0 : chunk;
    const float *kc = k + (size_t)c0 * width, *qc = q + (size_t)c0 * width;
    float dec = 1.0f;
    for (int t = 0; t < count; ++t) {
      dec = dec * decay[c0 + t];
      cumulative[t] = dec;
      products[t][t] = 1.0f;
      for (int j = t - 1; j >= 0; --j) products[t][j] = products[t][j + 1] * decay[c0 + j + 1];
      for (int j = 0; j < t; ++j) {
        float q_dot = po_float_dot(kc + (size_t)j * width, qc + (size_t)t * width, (size_t)width);
        float k_dot = po_float_dot(kc + (size_t)j * width, kc + (size_t)t * width, (size_t)width);
        cross_query[t][j] = products[t][j] * q_dot;
        cross_key[t][j] = products[t][j] * k_dot;
      }
      cross_query[t][t] = products[t][t] *
          po_float_dot(kc + (size_t)t * width, qc + (size_t)t * width, (size_t)width);
    }
    memcpy(prev, state, (size_t)rows * width * sizeof(float));
    const float last_cum = cumulative[count - 1];
    for (int r = 0; r < rows; ++r) {
      const float *s = prev + (size_t)r * width;
      for (int t = 0; t < count; ++t) {
        float key_dot = po_float_dot(s, kc + (size_t)t * width, (size_t)width);
        float query_dot = po_float_dot(s, qc + (size_t)t * width, (size_t)width);
        float predicted = cumulative[t] * key_dot;
        for (int j = 0; j < t; ++j) predicted = predicted + cross_key[t][j] * deltas[j];
        deltas[t] = (v[(size_t)(c0 + t) * rows + r] - predicted) * beta[c0 + t];
        float value = cumulative[t] * query_dot;
        for (int j = 0; j <= t; ++j) value = value + cross_query[t][j] * deltas[j];
        out[(size_t)(c0 + t) * rows + r] = value * scale;
      }
      float *m = state + (size_t)r * width;
      for (int i = 0; i < width; ++i) m[i] = last_cum * s[i];
      for (int j = 0; j < count; ++j) {
        float sd = products[count - 1][j] * deltas[j];
        const float *kj = kc + (size_t)j * width;
        for (int i = 0; i < width; ++i) m[i] = m[i] + sd * kj[i];
      }
    }
    for (size_t i = 0; i < (size_t)rows * width; ++i)
      if (!isfinite(state[i])) {
        free(prev);
        return PO_E_NONFINITE;
      }
  }
  free(prev);
  return PO_OK;
}

/* reference src/graph.rs:4956-5390 recurrent_attention (Source) */
static int recurrent_attention(po_qwen35 *m, int l, int threads) {
  const po_qwen35_config *c = &m->cfg;
  const int S = c->ssm_state, kw = key_width(c), vw = value_width(c), ch = conv_channels(c);
  const int K = c->conv_kernel, hist = K - 1;
  const void *ws[4] = {W(m, l, PO_W_QKV), W(m, l, PO_W_GATE), W(m, l, PO_W_BETA),
                       W(m, l, PO_W_ALPHA)};
  int rows[4] = {ch, vw, c->ssm_values, c->ssm_values};
  float *outs[4] = {m->mixed, m->zgate, m->beta, m->alpha};
  int st = project_group(m, m->normalized, c->hidden, 4, ws, rows, outs, threads);
  if (st) return st;
  const float *coef = (const float *)W(m, l, PO_W_CONV);
  const float *history = m->conv[l];
  for (int j = 0; j < ch; ++j) {
    float projected = m->mixed[j];
    const float *hj = history + (size_t)j * hist;
    const float *cj = coef + (size_t)j * K;
    float sum = 0.0f;
    for (int i = 0; i < hist; ++i) sum = sum + hj[i] * cj[i];
    sum = sum + projected * cj[hist];
    m->mixed[j] = sum;
    float *nj = m->next_conv + (size_t)j * hist;
    for (int i = 0; i + 1 < hist; ++i) nj[i] = hj[i + 1];
    if (hist > 0) nj[hist - 1] = projected;
  }
  for (int j = 0; j < ch; ++j) m->mixed[j] = po_silu(m->mixed[j]);
  for (int h = 0; h < 2 * kw / S; ++h) po_l2_norm(m->mixed + (size_t)h * S, (size_t)S, c->eps);
  const float *dt = (const float *)W(m, l, PO_W_DT_BIAS);
  const float *a = (const float *)W(m, l, PO_W_SSM_A);
  const float *nw = (const float *)W(m, l, PO_W_SSM_NORM);
  for (int h = 0; h < c->ssm_values; ++h) {
    const int kh = h % c->ssm_groups;
    const float *q = m->mixed + (size_t)kh * S;
    const float *k = m->mixed + kw + (size_t)kh * S;
    const float *v = m->mixed + 2 * kw + (size_t)h * S;
    float decay;
    if ((st = po_recurrent_decay(m->alpha[h], dt[h], a[h], &decay))) return st;
    const float beta = po_sigmoid(m->beta[h]);
    float *o = m->attended + (size_t)h * S;
    if ((st = po_gdn_head_step(m->matrix[l] + (size_t)h * S * S,
                               m->next_matrix + (size_t)h * S * S, q, k, v, decay, beta, S, S, o)))
      return st;
    /* reference src/kernels.rs:3589-3625 rms_norm_swiglu (Source) */
    float normed[512];
    if ((st = po_rms_norm(o, nw, (size_t)S, c->eps, normed))) return st;
    const float *z = m->zgate + (size_t)h * S;
    for (int i = 0; i < S; ++i) o[i] = normed[i] * po_silu(z[i]);
  }
  const void *wo[1] = {W(m, l, PO_W_SSM_OUT)};
  int ro[1] = {c->hidden};
  float *oo[1] = {m->attn_out};
  if ((st = project_group(m, m->attended, vw, 1, wo, ro, oo, threads))) return st;
  memcpy(m->matrix[l], m->next_matrix, (size_t)c->ssm_values * S * S * 4);
  memcpy(m->conv[l], m->next_conv, (size_t)ch * hist * 4);
  return PO_OK;
}

int po_qwen35_step(po_qwen35 *m, uint32_t token, float *logits, int threads) {
  const po_qwen35_config *c = &m->cfg;
  if ((int)token >= c->vocab || m->position >= c->context) return PO_E_INVALID;
  const size_t row_bytes = (size_t)c->hidden / 256 * block_bytes_of(c);
  int st;
  /* embedding row (reference src/graph.rs:3758 row_into) */
  if (c->weight_kind == 35)
    st = po_tq2_decode(m->embd + (size_t)token * row_bytes, (size_t)c->hidden / 256, m->hidden);
  else
    st = po_q2k_decode(m->embd + (size_t)token * row_bytes, (size_t)c->hidden / 256, m->hidden);
  if (st) return st;
  for (int l = 0; l < c->layers; ++l) {
    if ((st = po_rms_norm(m->hidden, (const float *)W(m, l, PO_W_ATTN_NORM), (size_t)c->hidden,
                          c->eps, m->normalized)))
      return st;
    st = po_qwen35_is_full_layer(c, l) ? full_attention(m, l, threads)
                                       : recurrent_attention(m, l, threads);
    if (st) return st;
    if ((st = po_add_rms_norm(m->hidden, m->attn_out, (const float *)W(m, l, PO_W_POST_NORM),
                              (size_t)c->hidden, c->eps, m->normalized)))
      return st;
    const void *ws[2] = {W(m, l, PO_W_FFN_UP), W(m, l, PO_W_FFN_GATE)};
    int rows[2] = {c->ffn, c->ffn};
    float *outs[2] = {m->up, m->gate};
    if ((st = project_group(m, m->normalized, c->hidden, 2, ws, rows, outs, threads))) return st;
    for (int i = 0; i < c->ffn; ++i) m->up[i] = m->up[i] * po_silu(m->gate[i]);
    const void *wd[1] = {W(m, l, PO_W_FFN_DOWN)};
    int rd[1] = {c->hidden};
    float *od[1] = {m->down};
    if ((st = project_group(m, m->up, c->ffn, 1, wd, rd, od, threads))) return st;
    for (int i = 0; i < c->hidden; ++i) {
      m->hidden[i] = m->hidden[i] + m->down[i];
      if (!isfinite(m->hidden[i])) return PO_E_NONFINITE;
    }
  }
  if (logits) {
    if ((st = po_rms_norm(m->hidden, m->out_norm, (size_t)c->hidden, c->eps, m->normalized)))
      return st;
    const void *we[1] = {m->embd};
    int re[1] = {c->vocab};
    float *oe[1] = {logits};
    if ((st = project_group(m, m->normalized, c->hidden, 1, we, re, oe, threads))) return st;
  }
  m->position += 1;
  return PO_OK;
}

int po_greedy(const float *logits, size_t n, uint32_t *out) {
  if (n == 0 || !isfinite(logits[0])) return PO_E_INVALID;
  size_t best = 0;
  float maximum = logits[0];
  for (size_t i = 1; i < n; ++i) {
    if (!isfinite(logits[i])) return PO_E_INVALID;
    if (logits[i] > maximum) {
      maximum = logits[i];
      best = i;
    }
  }
  *out = (uint32_t)best;
  return PO_OK;
}

/* Last layer's scratch activations, for parity debugging:
 * 5 attended, 6 GDN gate projection, 7 FFN h = up*silu(gate), 8 FFN gate. */
const float *po_qwen35_scratch(const po_qwen35 *m, int which) {
  switch (which) {
    case 5: return m->attended;
    case 6: return m->zgate;
    case 7: return m->up;
    case 8: return m->gate;
    default: return NULL;
  }
}
