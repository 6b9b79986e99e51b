/*
 * qwen35_oracle.h -- CPU restatement of the reference's Qwen35 hybrid decoder
 * (full gated attention every `full_interval`-th layer, Gated DeltaNet in the
 * others) under the Source arithmetic contract.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and CPU baseline); never linked
 * into the product library.
 */
#ifndef QWEN35_ORACLE_H
#define QWEN35_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct po_qwen35_config {
  int32_t hidden, layers, heads, kv_heads, head_dim, rope_dim;
  int32_t rope_sections[4];
  float rope_base, eps;
  int32_t ffn, vocab, ssm_state, ssm_groups, ssm_values, conv_kernel, full_interval;
  int32_t context;
  uint32_t weight_kind; /* 35 (TQ2_0) or 10 (Q2_K) for every linear weight */
  uint32_t kv_policy;   /* 0: binary16 K/V; 1: Q8_0 records (see below);
                           2 rsq4, 3 rsq4vf, 4 rsq4k3v: the reference's
                           rotated scalar records (kvq_oracle.c), keys and
                           values per position [kv_heads][132 | 100 B]     */
} po_qwen35_config;

/* Q8_0 KV records (kv_policy 1; an addition of this build, not a reference
 * policy): each cached K or V row of one KV head (head_dim values, already
 * rounded to binary16 as the binary16 policy stores them) is split into
 * 32-value blocks coded by the reference's Source Q8_0 codec
 * (src/kernels.rs:552-617 q8_with_input<false,false,_>); the record is the
 * head_dim/32 binary16 scales followed by the head_dim codes
 * (272 bytes for head_dim 256).  Attention reads the dequantized values
 * scale*code (exact in binary32), for the current position too. */
#define PO_KV_Q8_0_RECORD(hd) ((hd) / 32 * 2 + (hd))

/* Per-layer weight slots (reference tensor names in comments,
 * src/graph.rs:3112-3238).  Linear weights are packed rows in the reference
 * byte layout; the rest are f32. */
enum {
  PO_W_ATTN_NORM = 0, /* blk.N.attn_norm.weight            [hidden]         */
  PO_W_POST_NORM,     /* blk.N.post_attention_norm.weight  [hidden]         */
  PO_W_FFN_GATE,      /* blk.N.ffn_gate.weight   hidden -> ffn              */
  PO_W_FFN_UP,        /* blk.N.ffn_up.weight     hidden -> ffn              */
  PO_W_FFN_DOWN,      /* blk.N.ffn_down.weight   ffn -> hidden              */
  PO_W_Q,             /* blk.N.attn_q.weight     hidden -> heads*hd*2       */
  PO_W_K,             /* blk.N.attn_k.weight     hidden -> kv*hd            */
  PO_W_V,             /* blk.N.attn_v.weight     hidden -> kv*hd            */
  PO_W_O,             /* blk.N.attn_output.weight heads*hd -> hidden        */
  PO_W_Q_NORM,        /* blk.N.attn_q_norm.weight [hd]                      */
  PO_W_K_NORM,        /* blk.N.attn_k_norm.weight [hd]                      */
  PO_W_QKV,           /* blk.N.attn_qkv.weight   hidden -> conv channels    */
  PO_W_GATE,          /* blk.N.attn_gate.weight  hidden -> value width      */
  PO_W_BETA,          /* blk.N.ssm_beta.weight   hidden -> ssm_values       */
  PO_W_ALPHA,         /* blk.N.ssm_alpha.weight  hidden -> ssm_values       */
  PO_W_SSM_OUT,       /* blk.N.ssm_out.weight    value width -> hidden      */
  PO_W_CONV,          /* blk.N.ssm_conv1d.weight [channels][conv_kernel]    */
  PO_W_DT_BIAS,       /* blk.N.ssm_dt.bias       [ssm_values]               */
  PO_W_SSM_A,         /* blk.N.ssm_a             [ssm_values]               */
  PO_W_SSM_NORM,      /* blk.N.ssm_norm.weight   [ssm_state]                */
  PO_W_PER_LAYER
};

typedef struct po_qwen35 po_qwen35;

/* globals[0] = token_embd.weight (packed, vocab rows, also the tied output
 * head), globals[1] = output_norm.weight (f32 [hidden]).  layers holds
 * layers*PO_W_PER_LAYER pointers (unused slots may be NULL).  Pointers are
 * borrowed for the model's lifetime. */
po_qwen35 *po_qwen35_create(const po_qwen35_config *cfg, const void *const *globals,
                            const void *const *layers);
void po_qwen35_destroy(po_qwen35 *m);
void po_qwen35_reset(po_qwen35 *m);
int po_qwen35_is_full_layer(const po_qwen35_config *cfg, int layer);
/* One token through every layer; logits (vocab floats) when non-NULL.
 * threads = row-parallel workers for each projection. */
int po_qwen35_step(po_qwen35 *m, uint32_t token, float *logits, int threads);
int32_t po_qwen35_position(const po_qwen35 *m);
/* Copies of the recurrent/KV state for parity checks.  conv: [channels][k-1]
 * history; matrix: [ssm_values][ssm_state rows][ssm_state cols];
 * keys/values: [position][kv*hd] binary16 bits. */
const float *po_qwen35_conv_state(const po_qwen35 *m, int layer);
const float *po_qwen35_matrix_state(const po_qwen35 *m, int layer);
const uint16_t *po_qwen35_keys(const po_qwen35 *m, int layer);
const uint16_t *po_qwen35_values(const po_qwen35 *m, int layer);
const float *po_qwen35_hidden(const po_qwen35 *m);
const float *po_qwen35_scratch(const po_qwen35 *m, int which);

/* Overwrite one layer's recurrent or cached state with `bytes` bytes from
 * src (which: 0 conv [channels][k-1], 1 matrix [values][S][S], 2 keys,
 * 3 values -- the first `bytes` of the [context] cache rows), and set the
 * position: a checker continues decoding from a state produced elsewhere.
 * Returns PO_E_INVALID for a layer of the wrong kind or an oversize copy. */
int po_qwen35_load_state(po_qwen35 *m, int layer, int which, const void *src, size_t bytes);
int po_qwen35_set_position(po_qwen35 *m, int32_t position);

/* Greatest finite logit, lowest index on ties (reference src/runtime.rs:2630). */
int po_greedy(const float *logits, size_t n, uint32_t *out);

/* ---- op-level primitives (also used by the model) --------------------- */
/* One GDN decode step of one head (Source rows, reference src/graph.rs:801-822,
 * 5191-5343): prev/next [rows][width]; out[rows] = o_r * (1/sqrt(width)). */
int po_gdn_head_step(const float *prev, float *next, const float *q, const float *k,
                     const float *v, float decay, float beta, int rows, int width,
                     float *out);
/* Exact sequential prefill of one head over T tokens (reference
 * src/graph/prefill_gdn.rs:143-216): q,k,v [T][width], decay/beta [T],
 * out [T][rows]; state updated in place. */
int po_gdn_head_prefill_exact(float *state, const float *q, const float *k, const float *v,
                              const float *decay, const float *beta, int T, int rows,
                              int width, float *out);
/* Chunkwise prefill (reference src/graph/prefill_gdn.rs:223-456 head_into,
 * generalised from its 32-token bound to `chunk` <= 64 tokens). */
int po_gdn_head_prefill_chunked(float *state, const float *q, const float *k, const float *v,
                                const float *decay, const float *beta, int T, int rows,
                                int width, int chunk, float *out);
/* RoPE frequencies (reference src/graph.rs:6406-6437) for text position p. */
void po_rope_frequencies(const po_qwen35_config *cfg, int position, float *cos_sin);

#ifdef __cplusplus
}
#endif

#endif
