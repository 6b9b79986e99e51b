/*
 * prism_oracle.h -- CPU restatement of the prism-inference reference arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 kernels and the timed CPU baseline in bench.py.  It is never linked
 * into, loaded by, or called from the product library (libprism_b200.so).
 *
 * Every function restates the reference's "Source" arithmetic contract
 * (the contract any synthetic / random-init model receives, reference
 * src/graph.rs:3085-3110): binary32 products, binary64 sums where the
 * reference sums in binary64, separate (unfused) multiply and add, and
 * ties-to-even Q8_K rounding of the rounded binary32 product.
 *
 * Parity pin: the codec and dot functions reproduce the reference's golden
 * fixtures bit for bit (the JSON files under tests/golden, extracted from the reference's
 * tests/fixtures/upstream-tquants.json, upstream-kquants.json and
 * swift-q8k-parity.json by tests/golden/make_golden.py).
 */
#ifndef PRISM_ORACLE_H
#define PRISM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (0 = ok).  Errors mirror the reference's `invalid(...)` sites. */
#define PO_OK 0
#define PO_E_INVALID 1
#define PO_E_NONFINITE 3

/* Native Q8_K activation block, reference tools/ternary/src/lib.rs:27-39
 * (repr(C), 292 bytes: f32 scale, 256 x i8, 16 x i16 group sums). */
typedef struct po_q8k_block {
  float scale;
  int8_t values[256];
  int16_t sums[16];
} po_q8k_block;

/* Q8_0 record as stored by the KV cache extension: fp16 scale + 32 codes
 * (34 bytes), built by the reference's Source Q8_0 codec
 * (src/kernels.rs:552-617 with PINNED=false, NATIVE_SCALE=false). */
typedef struct po_q8_0_block {
  uint16_t d;
  int8_t values[32];
} po_q8_0_block;

/* ---- pinned (Swift) arithmetic variants (pinned_oracle.c) ------------- */
/* The reference's PinnedSwift GDN dot / scaled update, attention dot,
 * vector exponential, softmax and RoPE, for checking its native captures. */
float po_pinned_gdn_dot(const float *a, const float *b, size_t n);
int po_pinned_gdn_add_scaled(float *target, const float *input, float scale, size_t n);
int po_pinned_gdn_prefill(float *state, const float *q, const float *k, const float *v,
                          const float *decay, const float *beta, int batch, int tokens, int heads,
                          int key_heads, int d, float *out);
int po_pinned_attention_dot(const float *values, const float *weights, size_t n, float *out);
float po_vector_exp(float value);
int po_pinned_softmax(float *scores, size_t n, int round_f16);
/* x: n values, heads of `head`; cos_sin: rotary/2 (cos, sin) pairs. */
int po_pinned_rope(float *x, size_t n, int head, int rotary, const float *cos_sin, int in_place);
int po_source_rope(float *x, size_t n, int head, int rotary, const float *cos_sin);

/* ---- seeded synthetic weights (synth_inputs.c) ------------------------ */
/* rows x cols/256 packed blocks of kind 35 (TQ2_0) or 10 (Q2_K) in the
 * reference byte layout, the same bytes as the product library's seeded
 * generator for the same (seed, stream, lo, hi). */
int po_synth_weights(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t seed,
                     uint64_t stream, float lo, float hi, uint8_t *out);

/* ---- binary16 ------------------------------------------------------- */
float po_half_to_float(uint16_t h);
uint16_t po_float_to_half(float f);
float po_round_f16(float f);

/* ---- activation quantizers ------------------------------------------ */
int po_q8k_quantize(const float *x, size_t n, int pinned, po_q8k_block *out);
int po_q8_0_quantize(const float *x, size_t n, po_q8_0_block *out);

/* ---- TQ2_0 (ggml type 35, 66 B / 256 weights) ----------------------- */
int po_tq2_decode(const uint8_t *blocks, size_t nblocks, float *out);
int po_tq2_quantize(const float *x, size_t n, uint8_t *out);
int po_tq2_block_dots(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
                      int32_t *ints);
int po_tq2_dot(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
               float *out);

/* ---- Q2_K (ggml type 10, 84 B / 256 weights) ------------------------ */
int po_q2k_decode(const uint8_t *blocks, size_t nblocks, float *out);
int po_q2k_block_dots(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
                      int32_t *isum, int32_t *msum);
int po_q2k_dot(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
               float *out);

/* ---- row-parallel matvec (CPU baseline) ----------------------------- */
/* y[r] = dot(row r, a) for kind 35 or 10; rows split into contiguous
 * chunks over `threads` workers as reference RowParallelism::fill does
 * (src/kernels/parallel_rows.rs:507-542,602-628).  First error in row
 * order wins; output is zero-filled on error. */
int po_matvec(uint32_t kind, const uint8_t *w, size_t rows, size_t cols,
              const po_q8k_block *a, float *y, int threads);
int po_block_bytes(uint32_t kind);

/* Multi-token projection y[t][r] = dot(row r, Q8_K(x[t])) for `tokens`
 * rows of x [tokens][cols]: each token quantized once, each weight row
 * shared across tiles of 32 tokens (reference src/kernels/prefill.rs:26,
 * 48-87), rows split over `threads` workers in contiguous chunks. */
int po_project_tokens(uint32_t kind, const uint8_t *w, size_t rows, size_t cols,
                      const float *x, size_t tokens, int pinned, float *y, int threads);

/* ---- PQ2 (type 142, 34 B / 128 weights) and PTQ1 (type 143, 28 B) --
 * (packed_oracle.c).  Decoders give the 128 weights of a block (-1..2);
 * dots follow the reference's Q8_K and Q8_0 contracts; the matvec
 * quantizes x by the contract of (kind, cols) and dots every row. */
void po_pq2_values(const uint8_t *block, int16_t *out);
void po_ptq1_values(const uint8_t *block, int16_t *out);
int po_packed_block_bytes(uint32_t kind);
int po_packed_uses_q8k(uint32_t kind, size_t cols);
int po_pq2_dot_q8k(const uint8_t *w, size_t nblocks, const po_q8k_block *a, int fused,
                   float *out);
int po_packed_dot_q8(uint32_t kind, const uint8_t *w, size_t nblocks, const po_q8_0_block *a,
                     float *out);
int po_packed_matvec(uint32_t kind, const uint8_t *w, size_t rows, size_t cols, const float *x,
                     int fused, float *y);
int po_packed_row(uint32_t kind, const uint8_t *w, size_t cols, size_t r, float *out);

/* ---- float primitives (Source contract) ----------------------------- */
float po_float_dot(const float *a, const float *b, size_t n);
float po_f16_dot(const float *a, const uint16_t *b, size_t n);
float po_expf(float x);
float po_logf(float x);
float po_sinf(float x);
float po_cosf(float x);
float po_silu(float v);
float po_sigmoid(float v);
int po_recurrent_decay(float alpha, float time_bias, float decay_weight,
                       float *out);
int po_rms_norm(const float *x, const float *w, size_t n, float eps,
                float *out);
int po_add_rms_norm(float *values, const float *delta, const float *w,
                    size_t n, float eps, float *out);
void po_l2_norm(float *x, size_t n, float eps);
int po_softmax_round_f16(float *v, size_t n);

/* ---- TQ1_0 (34) and Q3_K..Q6_K (11-14) (kquant_oracle.c) ------------ */
int po_ext_block_bytes(uint32_t kind);
int po_ext_decode(uint32_t kind, const uint8_t *blocks, size_t nblocks, float *out);
int po_ext_block_ints(uint32_t kind, const uint8_t *w, const po_q8k_block *a, size_t nblocks,
                      int32_t *lanes, int32_t *msum);
int po_ext_dot(uint32_t kind, const uint8_t *w, const po_q8k_block *a, size_t nblocks,
               float *out);
int po_tq_quantize(uint32_t kind, const float *x, size_t n, uint8_t *out);

/* ---- batched gated-delta op with snapshots / replay (gdn_op_oracle.c) -- */
typedef struct po_gdn_op {
  uint32_t width, heads, tokens, sequences;
  uint32_t q_heads, k_heads, q_sequences, k_sequences;
  uint32_t gate_width;  /* 1 or width */
  uint32_t snapshots;
  int32_t raw, replay;
  uint32_t state_rows;  /* rows of the state table */
  uint32_t record_banks;
  uint64_t record_bank_elems, records_len;
} po_gdn_op;
int po_gdn_delta_values(const po_gdn_op *op, const float *q, const float *k, const float *v,
                        const float *gate, const float *beta, const float *table,
                        const int32_t *rows, const float *bias, const float *weight,
                        const float *records, const int32_t *control, float *out);
size_t po_gdn_delta_values_outputs(const po_gdn_op *op);

/* ---- rotated scalar KV codec, rsq (kvq_oracle.c) -------------------- */
uint64_t po_kvq_splitmix(uint64_t *state);
void po_kvq_levels(int levels, float *out);
int po_kvq_record_bytes(int bits);
int po_kvq_encode(int bits, uint64_t seed, int version, const float *input, uint8_t *out);
int po_kvq_rotate(int bits, uint64_t seed, const float *input, float *out);
int po_kvq_inverse(int bits, uint64_t seed, float *inout);
int po_kvq_score(int bits, const float *rotated_query, const uint8_t *rec, float *out);
int po_kvq_accumulate(int bits, const uint8_t *rec, float weight, float *out);
int po_kvq_decode(int bits, uint64_t seed, const uint8_t *rec, float *out);
int po_kvq_attend_head(int kbits, uint64_t kseed, int vbits, uint64_t vseed, const float *query,
                       const uint8_t *keys, const uint8_t *values, size_t n, float attn_scale,
                       const float *gate, float *out);

#ifdef __cplusplus
}
#endif

#endif
