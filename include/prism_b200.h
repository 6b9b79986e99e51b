/*
 * prism_b200.h -- C ABI of the B200 (sm_100a) quantized projection executor.
 *
 * This is the drop-in boundary for prism-inference's quantized decode path.
 * Each entry point replaces one method of the reference's projection
 * executor seam, `trait Pq2ProjectionExecutor`
 * (reference src/kernels/projection.rs:16-350), or a CPU kernel the seam
 * does not cover yet (cited per function).  A Rust host crate binds these
 * symbols with `extern "C"` declarations.
 *
 * Conventions
 *  - Plain C types only; no CUDA or framework types.  `stream` arguments
 *    are a `cudaStream_t` passed as `void*` (NULL = the executor's stream).
 *  - Entry points without `_device` take HOST pointers and are synchronous:
 *    they copy inputs in, run, copy outputs out and return a status.  The
 *    `_device` variants take DEVICE pointers and only enqueue work; their
 *    device-side errors surface at the next prism_b200_executor_sync().
 *  - Status codes: PRISM_B200_OK (0) or one of PRISM_B200_E_*.  A device-side
 *    failure (nonfinite output, bounded-wait timeout) is terminal for the
 *    executor, as in the reference: no CPU replay; the output is zero-filled;
 *    the executor reports PRISM_B200_E_FAULTED until
 *    prism_b200_executor_reset().  Argument errors are decided before any
 *    submission and leave the executor usable.
 *  - One executor = one CUDA device + one stream.  Not thread-safe: callers
 *    serialise, as the reference's `&mut self` executor scope does.
 *  - Caller-owned buffers are never retained after a call returns
 *    (reference src/kernels/projection.rs:10-13).
 */
#ifndef PRISM_B200_H
#define PRISM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PRISM_B200_ABI_VERSION 1

/* ---- status codes --------------------------------------------------- */
#define PRISM_B200_OK 0
#define PRISM_B200_E_INVALID 1     /* malformed arguments / extents          */
#define PRISM_B200_E_UNSUPPORTED 2 /* tensor kind or geometry not served     */
#define PRISM_B200_E_NONFINITE 3   /* nonfinite scale, activation or output  */
#define PRISM_B200_E_DEVICE 4      /* CUDA runtime / allocation failure      */
#define PRISM_B200_E_TIMEOUT 5     /* a bounded device wait expired          */
#define PRISM_B200_E_FAULTED 6     /* executor closed by an earlier failure  */

/* ---- tensor kinds (ggml / Prism type ids) --------------------------- */
#define PRISM_B200_KIND_Q2_K 10
#define PRISM_B200_KIND_Q8_K 15
#define PRISM_B200_KIND_TQ2_0 35
/* The rest of the reference's Q8_K activation contract (reference
 * src/kernels.rs:1653-1674): TQ1_0 54 B and Q3_K 110, Q4_K 144, Q5_K 176,
 * Q6_K 210 B per 256 weights, in the upstream ggml byte layouts
 * (src/kernels/tquants.rs, src/kernels/kquants.rs).  Kept as uploaded and
 * projected by prism_b200_project, _project_device and _project_f32. */
#define PRISM_B200_KIND_TQ1_0 34
#define PRISM_B200_KIND_Q3_K 11
#define PRISM_B200_KIND_Q4_K 12
#define PRISM_B200_KIND_Q5_K 13
#define PRISM_B200_KIND_Q6_K 14
/* The reference's own packed ternary formats (reference src/kernels.rs:
 * 85-86, 178-183): 128 weights per block, PQ2 in 34 bytes (binary16 scale,
 * then 2-bit codes), PTQ1 in 28 bytes (base-3 digits, then the scale). */
#define PRISM_B200_KIND_PQ2 142
#define PRISM_B200_KIND_PTQ1 143

/* Native Q8_K activation block (reference tools/ternary/src/lib.rs:27-39):
 * repr(C), 292 bytes. */
typedef struct prism_b200_q8k_block {
  float scale;
  int8_t values[256];
  int16_t sums[16];
} prism_b200_q8k_block;

/* One Q8_0 activation block (the reference's Q8Block, src/kernels.rs:
 * 524-535): scale (binary16-rounded) and scaled code sum as binary32, then
 * 32 codes; 40 bytes. */
typedef struct prism_b200_q8_block {
  float scale;
  float sum;
  int8_t values[32];
} prism_b200_q8_block;

/* A packed weight tensor in the reference's byte layout
 * (reference src/model.rs:184-196 `Tensor`): `cols` = dimensions[0] (K),
 * `rows` = product of the remaining dimensions, row-major rows of
 * cols/256 blocks.  `data` is a host pointer of rows*cols/256*block bytes. */
typedef struct prism_b200_tensor {
  uint32_t kind;
  uint64_t cols;
  uint64_t rows;
  const void *data;
} prism_b200_tensor;

typedef struct prism_b200_executor prism_b200_executor;
typedef struct prism_b200_weight prism_b200_weight;

/* ---- executor lifetime ---------------------------------------------- */

/* Create an executor on CUDA device `device` with its own stream. */
int prism_b200_executor_create(int device, prism_b200_executor **out);
void prism_b200_executor_destroy(prism_b200_executor *ex);

/* Stable arithmetic/placement identity string
 * (reference src/kernels/projection.rs:18 `identity`). */
const char *prism_b200_executor_identity(const prism_b200_executor *ex);

/* Copies the last error message (NUL-terminated, truncated to `len`);
 * returns the full message length. */
size_t prism_b200_executor_last_error(const prism_b200_executor *ex, char *buf,
                                      size_t len);

/* Wait for all enqueued work; returns the first device-side status. */
int prism_b200_executor_sync(prism_b200_executor *ex);

/* The executor's own stream (a cudaStream_t), for callers that order their
 * work or timing events against it. */
void *prism_b200_executor_stream(const prism_b200_executor *ex);

/* Clear a FAULTED executor (drops its sticky status, zeroes its scratch
 * counters).  The caller restarts its scope, as the reference reopens a
 * closed decoder scope. */
int prism_b200_executor_reset(prism_b200_executor *ex);

/* Eligibility from geometry alone, before any submission
 * (reference src/kernels/projection.rs:41-46 `supports`).  Returns 1 when
 * the tensor's kind is TQ2_0, Q2_K, TQ1_0 or Q3_K..Q6_K and cols is a
 * positive multiple of 256, or PQ2 or PTQ1 and cols is a positive multiple
 * of 128. */
int prism_b200_executor_supports(const prism_b200_executor *ex,
                                 const prism_b200_tensor *tensor);

/* Submission count of one projection (reference
 * src/kernels/projection.rs:28-35 `operation_count`): the number of
 * 32-row x 256-column work units (PQ2 / PTQ1: rows x 128-column blocks;
 * TQ1_0, Q3_K..Q6_K: rows x 256-column blocks), or -1 when unsupported. */
int64_t prism_b200_executor_operation_count(const prism_b200_executor *ex,
                                            const prism_b200_tensor *tensor);

/* ---- resident weights ----------------------------------------------- */

/* Validate (finite fp16 scales, exact extents) and upload a weight once;
 * it stays resident in HBM until released: TQ2_0 and Q2_K in the executor's
 * tiled layout, PQ2, PTQ1, TQ1_0 and Q3_K..Q6_K as uploaded.  Mirrors the
 * resident tiles of the reference's DSP executor (reference
 * docs/inference-efficiency.md:266-277).  PQ2 and PTQ1 weights serve
 * prism_b200_project, _project_device, _project_q8 and _project_f32; TQ1_0
 * and Q3_K..Q6_K the same but _project_q8 (they take Q8_K); the other
 * projections refuse them with PRISM_B200_E_UNSUPPORTED. */
int prism_b200_weight_upload(prism_b200_executor *ex,
                             const prism_b200_tensor *tensor,
                             prism_b200_weight **out);
void prism_b200_weight_release(prism_b200_weight *w);

/* ---- projections ---------------------------------------------------- */

/* y = W x over already quantized Q8_K activations
 * (reference src/kernels/projection.rs:48-60 `project`; per-row arithmetic
 * of src/kernels/tquants.rs:270-287, src/kernels/kquants.rs:346-420 and,
 * for PQ2, src/kernels.rs:941-959).  `activation` holds cols/256 blocks;
 * `out` receives rows floats.  `fused` selects the PQ2 fused multiply-add
 * contract and has no effect on TQ2_0 / Q2_K, whose reference dots have one
 * order.  PTQ1, and PQ2 whose cols is not a multiple of 256, take Q8_0
 * activations instead: PRISM_B200_E_UNSUPPORTED, `out` zero-filled. */
int prism_b200_project(prism_b200_executor *ex, const prism_b200_weight *w,
                       const prism_b200_q8k_block *activation, int fused,
                       float *out);
int prism_b200_project_device(prism_b200_executor *ex,
                              const prism_b200_weight *w,
                              const void *activation_dev, int fused,
                              float *out_dev, void *stream);

/* Quantize x (n = cols floats) to Q8_K on the device and project
 * (reference src/kernels.rs:1935-1987 `MatvecScratch::prepare` followed by
 * `PreparedMatvec::matvec_into`; src/kernels/projection.rs:95-107
 * `project_f32`).  `pinned` selects the pinned fused Q8_K rounding
 * (reference src/kernels.rs:421-428); 0 is the Source contract.  PQ2 and
 * PTQ1 quantize by their activation contract (Q8_K for PQ2 with a multiple
 * of 256 columns, else Q8_0) and dot unfused; `pinned` is refused there. */
int prism_b200_project_f32(prism_b200_executor *ex, const prism_b200_weight *w,
                           const float *x, int pinned, float *out);

/* Sibling projections sharing one activation vector, quantized once
 * (reference src/kernels/projection.rs:112-131 `project_f32_group`;
 * src/graph.rs:1869 `project_group_into_with_executor`). */
int prism_b200_project_f32_group(prism_b200_executor *ex, size_t count,
                                 const prism_b200_weight *const *weights,
                                 const float *x, int pinned,
                                 float *const *outs);

/* One projection over a tile of token activations: x is [tokens][cols]
 * f32, out is [tokens][rows] f32 (reference src/kernels/projection.rs:
 * 137-153 `project_f32_tokens`, whose default runs `project_f32` per token;
 * the tiled prefill of src/kernels/prefill.rs:48-87 `dot_quantized_tile_row`
 * computes the same per-token dots).  Each token is quantized to Q8_K on
 * the device and every output equals what prism_b200_project_f32 gives for
 * that token alone, bit for bit.  The integer block dots run on the tensor
 * cores (tcgen05.mma kind::i8, 128 tokens x 128 rows per tile).
 * tokens <= 65536; x_dev 16-byte aligned. */
int prism_b200_project_f32_tokens(prism_b200_executor *ex, const prism_b200_weight *w,
                                  size_t tokens, const float *x, int pinned, float *out);
int prism_b200_project_f32_tokens_device(prism_b200_executor *ex, const prism_b200_weight *w,
                                         size_t tokens, const float *x_dev, int pinned,
                                         float *out_dev, void *stream);

/* ---- the rest of the executor trait ------------------------------------ */

/* Remaining submissions of a bounded session (reference
 * src/kernels/projection.rs:20-28 `operation_capacity`).  This executor has
 * no bounded session: always -1, the reference's `None` (opaque capacity). */
int64_t prism_b200_executor_operation_capacity(const prism_b200_executor *ex);

/* Direct F32 activations, one tensor or a sibling group sharing one input
 * (reference src/kernels/projection.rs:93-96 `supports_f32`, :110-113
 * `supports_f32_group`): kinds TQ2_0 / Q2_K with the geometry `supports`
 * accepts; a group of 1..4 tensors of one kind and one column count. */
int prism_b200_executor_supports_f32(const prism_b200_executor *ex,
                                     const prism_b200_tensor *tensor);
int prism_b200_executor_supports_f32_group(const prism_b200_executor *ex, size_t count,
                                           const prism_b200_tensor *const *tensors);

/* Q8_0 activations (reference src/kernels/projection.rs:62-90
 * `supports_q8` / `project_q8`), which the reference routes for PTQ1 and
 * odd-block PQ2 rows: `activation` holds cols/32 prism_b200_q8_block; per
 * 128-weight block the four groups' scale x integer dot are summed in
 * binary32, then output += scale x sum (src/kernels.rs:1043-1063).  TQ2_0
 * and Q2_K take Q8_K activations, so supports_q8 returns 0 for them and
 * project_q8 returns PRISM_B200_E_UNSUPPORTED (the reference trait's
 * default) with `out` zero-filled; the executor stays open.  `pinned`
 * (the native PTQ1 lane order) is refused the same way. */
int prism_b200_executor_supports_q8(const prism_b200_executor *ex,
                                    const prism_b200_tensor *tensor);
int prism_b200_project_q8(prism_b200_executor *ex, const prism_b200_weight *w,
                          const void *activation, int pinned, float *out);

/* 1: multi-token tiles run natively on the device (reference
 * src/kernels/projection.rs:270-274 `supports_tile_tokens`). */
int prism_b200_executor_supports_tile_tokens(const prism_b200_executor *ex);

/* Two or three sibling projections over a tile of tokens sharing one input
 * (reference src/kernels/projection.rs:158-210 `project_f32_pair_tokens`,
 * `project_f32_triple_tokens`): x is [tokens][cols], out_k [tokens][rows_k].
 * The tokens are quantized to Q8_K once and every weight runs on the
 * tensor cores over them; each token's outputs equal
 * prism_b200_project_f32_group's for that token, bit for bit.
 * weights[0..1] / [0..2] share kind and columns; tokens <= 65536. */
int prism_b200_project_f32_pair_tokens(prism_b200_executor *ex,
                                       const prism_b200_weight *const *weights, size_t tokens,
                                       const float *x, int pinned, float *out_a, float *out_b);
int prism_b200_project_f32_triple_tokens(prism_b200_executor *ex,
                                         const prism_b200_weight *const *weights, size_t tokens,
                                         const float *x, int pinned, float *out_a, float *out_b,
                                         float *out_c);

/* Fused ffn_gate + ffn_up + SwiGLU: out = up(x) * silu(gate(x)) (reference
 * src/kernels/projection.rs:212-260 `supports_f32_ffn_swiglu`,
 * `project_f32_ffn_swiglu`, `project_f32_ffn_swiglu_tokens`; SwiGLU as
 * src/graph.rs:121-131).  gate and up are [F][H] of one kind; out has F
 * values (per token: [tokens][F]).  One token runs as one projection
 * kernel over both weights; a token tile as two tensor-core GEMMs and an
 * elementwise kernel.  Both equal up/gate from prism_b200_project_f32_group
 * followed by the binary32 SwiGLU, bit for bit. */
int prism_b200_executor_supports_f32_ffn_swiglu(const prism_b200_executor *ex,
                                                const prism_b200_tensor *gate,
                                                const prism_b200_tensor *up);
int prism_b200_project_f32_ffn_swiglu(prism_b200_executor *ex, const prism_b200_weight *gate,
                                      const prism_b200_weight *up, const float *x, int pinned,
                                      float *out);
int prism_b200_project_f32_ffn_swiglu_tokens(prism_b200_executor *ex,
                                             const prism_b200_weight *gate,
                                             const prism_b200_weight *up, size_t tokens,
                                             const float *x, int pinned, float *out);

/* The full FFN chain for one token (reference src/kernels/projection.rs:
 * 262-293 `supports_f32_ffn_chain`, `project_f32_ffn_chain`):
 *   out = residual + down(Q8_K(up(x) * silu(gate(x))))
 * with `residual` optional (NULL: no add).  gate/up [F][H], down [H][F],
 * one kind.  `hadamard_block_size` must be 0 (no rotation): a rotated chain
 * returns PRISM_B200_E_UNSUPPORTED before any submission.  The token-tile
 * form is prism_b200_ffn_chain_tokens below. */
int prism_b200_executor_supports_f32_ffn_chain(const prism_b200_executor *ex,
                                               const prism_b200_tensor *gate,
                                               const prism_b200_tensor *up,
                                               const prism_b200_tensor *down);
int prism_b200_project_f32_ffn_chain(prism_b200_executor *ex, const prism_b200_weight *gate,
                                     const prism_b200_weight *up, const prism_b200_weight *down,
                                     const float *x, const float *residual,
                                     uint32_t hadamard_block_size, int pinned, float *out);

/* ---- FFN chain over tokens, one GPU or tensor-parallel ---------------- */

/* The full intra-layer FFN chain over a tile of token activations
 * (reference src/kernels/projection.rs:261-350
 * `project_f32_ffn_chain_tokens`, without a Hadamard block):
 *   out[m] = residual[m] + down(Q8_K(SwiGLU(gate(Q8_K(x_m)), up(Q8_K(x_m)))))
 * with SwiGLU(g, u) = u * silu(g) and `residual` optional.  gate and up are
 * [F][H] and down [H][F] resident weights of one kind.
 *
 * prism_b200_ffn_create prepares the chain for at most `max_tokens` tokens
 * per call.  With tp_size == 1 it computes every row on this GPU, bit for bit
 * the sequential chain.  With tp_size N > 1 this is rank `tp_rank` of N (one
 * process and GPU each): it keeps gate/up rows [r*F/N, (r+1)*F/N) and the
 * matching input blocks of down (F % (256 N) == 0), and the down projection's
 * partial sums are all-reduced over NVLink peer memory in rank order (within
 * a few binary32 ulps of the one-GPU chain).  Tensor-parallel ranks exchange
 * their 64-byte handles (prism_b200_ffn_exchange_handle, gathered in rank
 * order) and connect before the first call; every rank then calls with the
 * same token counts in the same order, like a collective.  A rank that stops
 * calling makes the others' waits expire (PRISM_B200_E_TIMEOUT). */
typedef struct prism_b200_ffn prism_b200_ffn;
int prism_b200_ffn_create(prism_b200_executor *ex, const prism_b200_weight *gate,
                          const prism_b200_weight *up, const prism_b200_weight *down,
                          uint32_t max_tokens, uint32_t tp_rank, uint32_t tp_size,
                          prism_b200_ffn **out);
void prism_b200_ffn_destroy(prism_b200_ffn *f);
int prism_b200_ffn_exchange_handle(const prism_b200_ffn *f, void *handle);
int prism_b200_ffn_connect(prism_b200_ffn *f, const void *handles);
int prism_b200_ffn_chain_tokens(prism_b200_ffn *f, size_t tokens, const float *x,
                                const float *residual, int pinned, float *out);
int prism_b200_ffn_chain_tokens_device(prism_b200_ffn *f, size_t tokens, const float *x_dev,
                                       const float *residual_dev, int pinned, float *out_dev,
                                       void *stream);

/* Q8_K activation quantization of n floats (n % 256 == 0)
 * (reference src/kernels.rs:463-522 `q8k_with_input`). */
int prism_b200_quantize_q8k(prism_b200_executor *ex, const float *x, size_t n,
                            int pinned, prism_b200_q8k_block *out);
int prism_b200_quantize_q8k_device(prism_b200_executor *ex, const float *x_dev,
                                   size_t n, int pinned, void *out_dev,
                                   void *stream);

/* f32 weights -> TQ1_0 (kind 34) or TQ2_0 (kind 35) blocks (reference
 * src/kernels/tquants.rs:288-336 `quantize`): per 256 values d = max |x|
 * stored as binary16, level = round-half-away(x * (1/d)) + 1.  `n` is a
 * positive multiple of 256; `out` receives n/256 blocks of 54 or 66 bytes.
 * A nonfinite input returns E_INVALID, a block maximum beyond binary16
 * E_NONFINITE (the device-side status rules above). */
int prism_b200_quantize_tq(prism_b200_executor *ex, uint32_t kind, const float *x, size_t n,
                           void *out);
int prism_b200_quantize_tq_device(prism_b200_executor *ex, uint32_t kind, const float *x_dev,
                                  size_t n, void *out_dev, void *stream);

/* The exact per-block integer dots of a projection, the parity observable
 * of the int32 contract (reference src/kernels/tquants.rs:220-245
 * `dot_tq2_block`; src/kernels/kquants.rs:162-200 `dot_q2_k_block`).
 * TQ2_0 writes rows*nb int32 (`ints`); Q2_K writes isum to `ints` and the
 * min-sum to `ints2` (each rows*nb int32).  Row-major [row][block]. */
int prism_b200_block_dots(prism_b200_executor *ex, const prism_b200_weight *w,
                          const prism_b200_q8k_block *activation,
                          int32_t *ints, int32_t *ints2);

/* ---- Gated DeltaNet recurrence --------------------------------------- */
/* For each sequence b < batch and value head h < heads (key head
 * h % key_heads), with state rows r = value channels:
 *   S_r <- decay*S_r; delta_r = (v_r - S_r.k)*beta; S_r += delta_r*k;
 *   out_r = (S_r.q)/sqrt(d)
 * (reference src/graph.rs:801-822 gdn_step_row_from, 5191-5343; batched as
 * src/backend/gdn.rs:24-300 with the gate given as its decay).  DEVICE
 * pointers, f32, d == 128:
 *   state [batch][heads][d][d] (updated in place)
 *   q, k  [batch][tokens][key_heads][d];  v, out [batch][tokens][heads][d]
 *   decay, beta [batch][tokens][heads]
 * decode_device runs one step (tokens = 1) with the reference's binary32
 * products summed in binary64; prefill_device runs `tokens` steps in chunks
 * of `chunk` (1..64) tokens with the chunkwise (WY) form of the reference's
 * src/graph/prefill_gdn.rs:223-456, in binary32, within 1e-3 + 1e-3*|ref|
 * of the sequential recurrence (the reference's stated chunkwise bound). */
int prism_b200_gdn_decode_device(prism_b200_executor *ex, int batch, int heads, int key_heads,
                                 int d, float *state, const float *q, const float *k,
                                 const float *v, const float *decay, const float *beta,
                                 float *out, void *stream);
int prism_b200_gdn_prefill_device(prism_b200_executor *ex, int batch, int tokens, int heads,
                                  int key_heads, int d, int chunk, float *state, const float *q,
                                  const float *k, const float *v, const float *decay,
                                  const float *beta, float *out, void *stream);

/* The reference's pinned ("Swift") GDN recurrence over device buffers in the
 * layout above (replaces src/kernels/pinned_gdn.rs:370-455 step_row_in_place
 * / step_row_tokens_from over a head, :853-973 step_head_tokens_in_place):
 * every state row stepped token by token -- row *= decay, dot_k = the pinned
 * 16-lane fused dot with the key (registers 0+2 and 1+3, then adjacent lane
 * pairs), delta = (v - dot_k) * beta, row += delta * key fused, out = the
 * pinned dot with the query * (1/sqrt(d)) -- bit for bit the reference's
 * scalar contract (which its NEON paths match).  d = 128.  A nonfinite dot
 * or state element reports PRISM_B200_E_NONFINITE at the next synchronising
 * call, where the reference returns its error. */
int prism_b200_gdn_prefill_pinned_device(prism_b200_executor *ex, int batch, int tokens,
                                         int heads, int key_heads, int d, float *state,
                                         const float *q, const float *k, const float *v,
                                         const float *decay, const float *beta, float *out,
                                         void *stream);

/* Same computation and arguments as prism_b200_gdn_prefill_device, but it
 * never allocates device memory.  This entry point has no counterpart in
 * the reference.  It is for hosts that cannot let a library allocate:
 * processes that reserved all device memory up front, and loops that cannot
 * take the device-wide synchronisation of an allocation.  Its chunk scratch
 * is a fixed array in the library's device image, of
 * PRISM_B200_GDN_STATIC_SCRATCH_BYTES; a call needing more
 * (batch x heads x ceil(tokens/chunk) x 35,328 bytes) fails with
 * PRISM_B200_E_INVALID before anything is enqueued.  The array is a device
 * module of its own: under CUDA's default lazy module loading it occupies
 * its 34 MiB on a device from the first call of this function there until
 * the context is destroyed (with CUDA_MODULE_LOADING=EAGER, on every device
 * the process initialises, called or not).  The first call in a context
 * loads that module and looks the array's address up, so make it before any
 * stream capture; the address is cached per context.  All callers on a
 * device share the array: calls whose kernels can overlap in time (other
 * streams, other executors) race and must be serialised by the caller. */
#define PRISM_B200_GDN_STATIC_SCRATCH_BYTES (34u * 1024u * 1024u)
int prism_b200_gdn_prefill_device_noalloc(prism_b200_executor *ex, int batch, int tokens,
                                          int heads, int key_heads, int d, int chunk,
                                          float *state, const float *q, const float *k,
                                          const float *v, const float *decay,
                                          const float *beta, float *out, void *stream);

/* ---- Qwen3.5-style hybrid decoder ----------------------------------- */
/* The reference's Qwen35 graph (reference src/graph.rs:2294 `Qwen35`,
 * `impl Decoder for Qwen35` src/graph.rs:5392-5580) on the device: every
 * `full_interval`-th layer is gated full attention over a KV cache, the
 * others Gated DeltaNet; the output head is tied to token_embd.weight.
 * Geometry fields mirror the reference's GGUF metadata keys
 * (src/graph.rs:2966-3056, `qwen35.*`). */
#define PRISM_B200_KV_F16 0
#define PRISM_B200_KV_Q8_0 1
/* The reference's rotated scalar KV policies (reference src/graph/
 * quantized_kv.rs:16-84 KvCachePolicy): every full-attention position is
 * stored as a record of the codec below per KV head, the current one too. */
#define PRISM_B200_KV_RSQ4 2    /* "rsq4": 4-bit keys and values            */
#define PRISM_B200_KV_RSQ4VF 3  /* "rsq4vf": values with fitted scales      */
#define PRISM_B200_KV_RSQ4K3V 4 /* "rsq4k3v": 4-bit keys, 3-bit values      */

typedef struct prism_b200_qwen35_config {
  uint32_t hidden;          /* qwen35.embedding_length            */
  uint32_t layers;          /* qwen35.block_count                 */
  uint32_t heads;           /* qwen35.attention.head_count        */
  uint32_t kv_heads;        /* qwen35.attention.head_count_kv     */
  uint32_t head_dim;        /* qwen35.attention.key_length        */
  uint32_t rope_dim;        /* qwen35.rope.dimension_count        */
  uint32_t rope_sections[4];/* qwen35.rope.dimension_sections     */
  float rope_base;          /* qwen35.rope.freq_base              */
  float eps;                /* qwen35.attention.layer_norm_rms_epsilon */
  uint32_t ffn;             /* qwen35.feed_forward_length         */
  uint32_t vocab;           /* rows of token_embd.weight          */
  uint32_t ssm_state;       /* qwen35.ssm.state_size              */
  uint32_t ssm_groups;      /* qwen35.ssm.group_count             */
  uint32_t ssm_values;      /* qwen35.ssm.time_step_rank          */
  uint32_t conv_kernel;     /* qwen35.ssm.conv_kernel             */
  uint32_t full_interval;   /* qwen35.full_attention_interval     */
  uint32_t context;         /* KV capacity in tokens (context_limit) */
  uint32_t kv_policy;       /* PRISM_B200_KV_*; the rotated policies
                               need context <= 32768                  */
  uint32_t weight_kind;     /* PRISM_B200_KIND_TQ2_0 or _Q2_K     */
} prism_b200_qwen35_config;

typedef struct prism_b200_model prism_b200_model;

int prism_b200_model_create(prism_b200_executor *ex, const prism_b200_qwen35_config *cfg,
                            prism_b200_model **out);
void prism_b200_model_destroy(prism_b200_model *m);

/* Bind a tensor by its reference name (src/graph.rs:3112-3238), e.g.
 * "token_embd.weight", "blk.3.ffn_down.weight".  Packed linear weights use
 * set_tensor (copied to HBM at once); f32 vectors (norms, ssm_conv1d,
 * ssm_dt.bias, ssm_a) use set_vector. */
int prism_b200_model_set_tensor(prism_b200_model *m, const char *name,
                                const prism_b200_tensor *t);
int prism_b200_model_set_vector(prism_b200_model *m, const char *name, const float *data,
                                size_t n);

/* Check every tensor is bound and build the step graphs. */
int prism_b200_model_finalize(prism_b200_model *m);

/* Clear the KV cache and recurrent state (position 0), as the reference's
 * Decoder::reset. */
int prism_b200_model_reset(prism_b200_model *m);
int64_t prism_b200_model_position(const prism_b200_model *m);

/* 1 when a step runs as one cooperative kernel (the dataflow step), 0 when
 * it runs as the per-phase kernel sequence.  Both give the same bits.  No
 * counterpart in the reference. */
int prism_b200_model_persistent(const prism_b200_model *m);

/* How a decode step runs, chosen at finalize: 2 = the dataflow kernel (one
 * cooperative launch per token; activations carry a per-step tag that their
 * consumers poll, weights stream through a shared-memory ring ahead of the
 * compute), the default wherever the model and device are eligible; 0 = the
 * per-phase kernel sequence in a CUDA graph (PRISM_B200_STEP=seq, or an
 * ineligible model).  -1 for a NULL model.  No counterpart in the
 * reference. */
int prism_b200_model_step_mode(const prism_b200_model *m);

/* For the kernel-sequence step, with PRISM_B200_TRACE=1 set before the
 * model is finalized: the last step's per-launch timelines in globaltimer
 * ns, 8 values per launch (per layer: projection group, GDN or attention,
 * out-projection, FFN pair, FFN down; then the LM head): CTA 0's [0] entry,
 * [1] grid dependency passed, [2] input staged, [3] first tile resident,
 * [4] its dots, [5] its chains, [6] exit, and [7] the last CTA's exit
 * (projections; GDN and attention stamp [0], [1], [6], [7]).
 * For the dataflow step (mode 2): CTA 0's stamps of the last
 * prism_b200_model_step_timings step, 16 values per phase (embedding, then
 * per layer three attention-side phases and the FFN pair, then the LM head),
 * globaltimer ns unless noted: [5] and [0] phase start, [6] descriptor read,
 * [7] phase end.  Projections: [1] input staged, [2] first batch's weights
 * resident, [3] its dots, [4] its chains, [8] before the weight wait, [9]
 * after it, [11] issue time of the batch's last piece, [12] pieces in the
 * batch (a count).  Attention: [1] inputs arrived, [2] query and key
 * normed, rotated and cached, [14] first K rows resident, [15] their
 * scores, [3] the share's scores, [4] every position's scores resident,
 * [10] softmax maximum, [11] exponentials, [12] share trees, [13] share
 * totals, [8] probabilities, [9] value sums.
 * Copies at most `count` values and returns how many (0 when no timeline
 * is recorded).  No counterpart in the reference. */
int64_t prism_b200_model_phase_trace(prism_b200_model *m, uint64_t *ns, size_t count);

/* Dataflow step only: every CTA's globaltimer stamps of the last
 * prism_b200_model_step_timings step, [phase][CTA][4] (grid = the SM
 * count): inputs arrived and input staged (projection phases, else 0),
 * phase end, and the end of the phase's first weight-batch planning
 * (projection phases, else 0), so that a phase's critical path (its slowest
 * CTA) can be read.  Copies at most `count` values and returns how many (0
 * for the kernel sequence).  No counterpart in the reference. */
int64_t prism_b200_model_phase_trace_ctas(prism_b200_model *m, uint64_t *ns, size_t count);

/* One token at the next position (reference Decoder::evaluate_finite_into,
 * src/graph.rs:5446).  `logits` (host, vocab floats) and `greedy` (the
 * reference's greedy selection, src/runtime.rs:2630) are optional. */
int prism_b200_model_evaluate(prism_b200_model *m, uint32_t token, float *logits,
                              uint32_t *greedy);

/* Ingest `n_prompt` tokens, then greedily generate `n_new` tokens entirely
 * on the device (reference Runtime::generate loop with greedy sampling,
 * src/runtime.rs:1944-2031); `out` receives the n_new tokens. */
int prism_b200_model_generate(prism_b200_model *m, const uint32_t *prompt, size_t n_prompt,
                              size_t n_new, uint32_t *out);

/* Enqueue `steps` device-driven decode steps on the model's stream without
 * waiting (each consumes the previous step's greedy token). */
int prism_b200_model_decode_async(prism_b200_model *m, size_t steps);

/* set_prompt places `n` prompt tokens at the next positions of the token
 * history; ingest_async then enqueues, without waiting, `n` ingestion steps
 * (no LM head, the reference's Decoder::ingest, src/lib.rs:229-247).  Decode
 * steps past the prompt consume the previous step's greedy token. */
int prism_b200_model_set_prompt(prism_b200_model *m, const uint32_t *tokens, size_t n);
int prism_b200_model_ingest_async(prism_b200_model *m, size_t n);

/* Batched prompt ingestion (replaces Decoder::ingest_block, src/lib.rs:229-247,
 * and its tiled override, src/graph.rs:5459-5461).  prefill_async enqueues,
 * without waiting, the ingestion of the `n` tokens that set_prompt placed at
 * the next positions: every layer processes up to 2048 tokens at once
 * (tensor-core projections over the tokens, the Gated DeltaNet recurrence
 * token after token with its state on chip, causal attention of each token
 * over its prefix).  The KV rows, recurrent and convolution state and
 * position it leaves are bit for bit those of `n` ingest steps.  Under the
 * rotated KV policies it runs those `n` ingest steps (the reference's tiled
 * prefill keeps their records bit for bit, tests/graph/quantized_kv.rs:
 * 164-260).  ingest_block is the reference's synchronous form: it rejects an empty
 * block, one longer than PRISM_B200_MAX_PREFILL_BLOCK_TOKENS or a token
 * outside the vocabulary before changing any state, then places, ingests and
 * waits, returning the device status. */
#define PRISM_B200_MAX_PREFILL_BLOCK_TOKENS 256u
int prism_b200_model_prefill_async(prism_b200_model *m, size_t n);
int prism_b200_model_ingest_block(prism_b200_model *m, const uint32_t *tokens, size_t n);

/* The model's own stream (a cudaStream_t). */
void *prism_b200_model_stream(const prism_b200_model *m);

/* Run one decode step (device-driven input, as decode_async) with CUDA
 * events between phases and report per-layer attention and FFN wall time,
 * the LM head and the whole step, in milliseconds (reference
 * src/graph/timing.rs TokenTimings).  Each array holds `layers` floats;
 * any pointer may be NULL.  The timed step runs without programmatic
 * dependent launch, so its total exceeds a graph step's. */
int prism_b200_model_step_timings(prism_b200_model *m, float *attention_ms, float *ffn_ms,
                                  float *head_ms, float *total_ms);

/* State readback for parity checks: which = 0 conv history [channels][k-1],
 * 1 recurrent matrix [values][S][S], 2 keys / 3 values [position][kv*hd]
 * binary16 (Q8_0: [position][kv][272 B]; rotated: [position][kv][132 or
 * 100 B] records), 4 hidden [hidden]; the last layer's activations: 5 attended,
 * 6 GDN gate projection, 7 FFN up*silu(gate), 9 logits.  Returns the byte
 * count written, or minus a status code. */
int64_t prism_b200_model_read_state(prism_b200_model *m, uint32_t layer, uint32_t which,
                                    void *out, size_t bytes);

/* ---- the batched gated-delta op (snapshots and replay) ------------------ */
/* The reference's ggml GDN backend op (reference src/backend/gdn.rs:24-300
 * CpuBackend::delta_values, operation 100, or 101 with `replay`).  Tensors
 * in ggml order (first index fastest), device pointers:
 *   q [width][q_heads][tokens][q_sequences], k [width][k_heads][tokens]
 *   [k_sequences] (head h reads q/k head h % q_heads, sequence s reads
 *   sequence s / (sequences / q_sequences)); v [width][heads][tokens]
 *   [sequences]; gate [gate_width = 1 or width][heads][tokens][sequences];
 *   beta [1][heads][tokens][sequences]; state table [width*width*heads]
 *   [state_rows]; rows (op 100, optional) the distinct table row of each
 *   sequence, else sequence s reads row s; bias, weight [heads] with `raw`
 *   (beta through the sigmoid, gate through weight * softplus(gate + bias));
 *   records [sequences][record_banks][record_bank_elems] and control
 *   [sequences][count, bank] with `replay`.
 * Per token: state *= exp(gate) (per column with per-column gates), delta =
 * (v - dot(S_row, k)) * beta, S_row += k * delta, out = dot(S_row, q) /
 * sqrt(width); dot sums exact binary64 products in column order.  `out`
 * (prism_b200_gdn_delta_values_outputs floats) receives the attention rows,
 * then the snapshot slots (slot tokens-1-t = the state after token t; slots
 * past the tokens keep their contents), or in replay the state after token
 * tokens - min(tokens, snapshots) and the later tokens' records
 * (delta[heads*width], keys[heads*width], decay[heads]).  Widths up to 128;
 * raw gates with replay are refused (the reference reads both from one
 * source).  Invalid rows, control or record extents are device-side errors
 * (E_INVALID at the next sync). */
typedef struct prism_b200_gdn_op {
  uint32_t width, heads, tokens, sequences;
  uint32_t q_heads, k_heads, q_sequences, k_sequences;
  uint32_t gate_width;
  uint32_t snapshots;
  int32_t raw, replay;
  uint32_t state_rows;
  uint32_t record_banks;
  uint64_t record_bank_elems, records_len;
} prism_b200_gdn_op;
size_t prism_b200_gdn_delta_values_outputs(const prism_b200_gdn_op *op);
int prism_b200_gdn_delta_values_device(prism_b200_executor *ex, const prism_b200_gdn_op *op,
                                       const float *q, const float *k, const float *v,
                                       const float *gate, const float *beta, const float *table,
                                       const int32_t *rows, const float *bias,
                                       const float *weight, const float *records,
                                       const int32_t *control, float *out, void *stream);

/* ---- GGUF model files --------------------------------------------------- */
/* The reference's model loading (reference src/model.rs:266-420 Model::load)
 * and Qwen35 geometry (src/graph.rs:2966-3100): gguf_open reads a GGUF file
 * (version 2 or 3) whole and checks its header, typed metadata, tensor table
 * and every tensor's extent and alignment (general.alignment, default 32);
 * tensor types are F32, F16 and the packed kinds above.  On failure `err`
 * (when given) receives the reason.  gguf_qwen35_config reads the
 * reference's `qwen35.*` keys (embedding_length, block_count,
 * attention.head_count[_kv], attention.key_length = value_length,
 * rope.dimension_count, rope.dimension_sections[4], rope.freq_base,
 * attention.layer_norm_rms_epsilon, feed_forward_length, ssm.state_size,
 * ssm.group_count, ssm.time_step_rank, ssm.conv_kernel, ssm.inner_size,
 * full_attention_interval (default 4) and, when present,
 * attention.recurrent_layers, which must follow that interval); the
 * vocabulary and weight kind come from token_embd.weight.  An untied
 * output.weight is refused (E_UNSUPPORTED): the head is the embedding.
 * model_load_gguf creates the model and binds every tensor by its GGUF
 * name (F32 / F16 tensors as vectors, packed ones as weights), then
 * finalizes it.  The file's bytes stay with the gguf handle; the model keeps
 * its own copies in HBM. */
typedef struct prism_b200_gguf prism_b200_gguf;
int prism_b200_gguf_open(const char *path, prism_b200_gguf **out, char *err, size_t err_len);
void prism_b200_gguf_close(prism_b200_gguf *g);
int64_t prism_b200_gguf_tensor_count(const prism_b200_gguf *g);
int prism_b200_gguf_tensor(const prism_b200_gguf *g, size_t index, const char **name,
                           uint32_t *type, uint64_t dims[4], uint32_t *ndims, const void **data,
                           uint64_t *bytes);
int prism_b200_gguf_qwen35_config(const prism_b200_gguf *g, uint32_t context, uint32_t kv_policy,
                                  prism_b200_qwen35_config *cfg, char *err, size_t err_len);
int prism_b200_model_load_gguf(prism_b200_executor *ex, const prism_b200_gguf *g,
                               uint32_t context, uint32_t kv_policy, prism_b200_model **out);

/* ---- decoder checkpoints ----------------------------------------------- */
/* The reference's Decoder::checkpoint / checkpoint_into / restore /
 * checkpoint_bytes (reference src/lib.rs:105,305-319; Qwen35 at
 * src/graph.rs:5483-5578).  A checkpoint is a device-resident copy of every
 * piece of state a later step reads: the KV rows of positions [0, p) (in the
 * model's KV policy), each GDN layer's recurrent matrix and convolution
 * history, the token history through the next input and the position.  It
 * restores only into the model that took it (the reference's provenance
 * check), on the same device; position 0 holds no layer payload and restores
 * as a reset.  checkpoint_into reuses the checkpoint's storage when it is
 * large enough.  The copies are device to device on the model's stream and
 * the calls wait for them. */
typedef struct prism_b200_checkpoint prism_b200_checkpoint;
int prism_b200_model_checkpoint(prism_b200_model *m, prism_b200_checkpoint **out);
int prism_b200_model_checkpoint_into(prism_b200_model *m, prism_b200_checkpoint *cp);
int prism_b200_model_restore(prism_b200_model *m, const prism_b200_checkpoint *cp);
int64_t prism_b200_checkpoint_bytes(const prism_b200_checkpoint *cp);
int64_t prism_b200_checkpoint_position(const prism_b200_checkpoint *cp);
void prism_b200_checkpoint_destroy(prism_b200_checkpoint *cp);

/* ---- batched serving -------------------------------------------------- */
/* Many sequences decoded together over one finalized model's resident
 * weights (its config, weights and KV policy).  Every step advances each of
 * the `sequences` by one token: the projections of all their tokens run as
 * tensor-core GEMMs, Gated DeltaNet and attention per (sequence, head) on
 * each sequence's own state and KV cache of `context` positions.  Each
 * sequence gets exactly what decoding it alone gives -- the reference's
 * weight-sharing batched evaluation contract (reference src/lib.rs:255-275
 * `evaluate_batch_into`); the reference server keeps one decoder per
 * sequence (reference server/src/native_backend).  Models under a rotated
 * KV policy are refused (E_UNSUPPORTED): they decode one sequence. */
typedef struct prism_b200_batch prism_b200_batch;
int prism_b200_batch_create(prism_b200_model *m, uint32_t sequences, uint32_t context,
                            prism_b200_batch **out);
void prism_b200_batch_destroy(prism_b200_batch *b);
/* Every sequence back to position 0 with empty state. */
int prism_b200_batch_reset(prism_b200_batch *b);
/* One step: tokens[sequences] in (host); greedy[sequences] (host, may be
 * NULL) receives each sequence's greedy next token, which also becomes its
 * input for prism_b200_batch_decode_async. */
int prism_b200_batch_step(prism_b200_batch *b, const uint32_t *tokens, uint32_t *greedy);
/* `steps` greedy steps on the batch's stream, each feeding the previous
 * step's greedy tokens back in (after at least one prism_b200_batch_step). */
int prism_b200_batch_decode_async(prism_b200_batch *b, size_t steps);
void *prism_b200_batch_stream(const prism_b200_batch *b);
/* Seeded synthetic context for benchmarks: every sequence at `position`
 * with random KV rows and recurrent/convolution state.  No counterpart in
 * the reference (it stands in for prompts the benchmark does not ingest). */
int prism_b200_batch_fill_context(prism_b200_batch *b, uint32_t position, uint64_t seed);
/* State of one sequence, as prism_b200_model_read_state (which 0..4).  On a
 * tensor-parallel batch, recurrent and KV state are this rank's heads. */
int64_t prism_b200_batch_read_state(prism_b200_batch *b, uint32_t seq, uint32_t layer,
                                    uint32_t which, void *out, size_t bytes);

/* Tensor-parallel batched serving over tp_size GPUs of one node, one
 * process (and one model holding the full weights) per GPU.  No counterpart
 * in the reference, which serves on host cores.  Rank `tp_rank` keeps a
 * column slice of every projection feeding a per-head or per-row operation
 * (attention query heads and their KV heads, Gated DeltaNet heads, 256-row
 * blocks of the FFN intermediate) and the output head's vocabulary rows.
 * attn_output, ssm_out and ffn_down, per `tp_mode`:
 *  - PRISM_B200_TP_EXACT: column-split as well.  Each rank's quantized head
 *    (FFN) outputs are gathered into every rank over NVLink peer memory,
 *    and each rank's slice of hidden rows is stored into every rank's
 *    hidden state (both fused into the producing kernels).  Bit-identical
 *    to the one-GPU batch and the oracle.
 *  - PRISM_B200_TP_ALLREDUCE: row-split (input blocks); the partial sums are
 *    all-reduced over peer memory (fused into the GEMM epilogue and the next
 *    RMSNorm, summed in rank order: every rank holds identical hidden
 *    states).  The cross-rank sums round differently from the reference's
 *    per-row chain, so outputs match the one-GPU batch to float rounding
 *    only, amplified by the Q8_K quantizers downstream.
 * All ranks pass the same tokens.  Connect before the first step: every
 * rank publishes its exchange handle (prism_b200_batch_exchange_handle), the
 * host gathers them in rank order (tp_size * PRISM_B200_EXCHANGE_HANDLE_BYTES)
 * and every rank passes the gathered array to prism_b200_batch_connect.  The
 * ranks' steps wait on one another (bounded: PRISM_B200_E_TIMEOUT when a
 * rank stops stepping).  tp_size 1 is prism_b200_batch_create. */
#define PRISM_B200_EXCHANGE_HANDLE_BYTES 64
#define PRISM_B200_TP_EXACT 0u
#define PRISM_B200_TP_ALLREDUCE 1u
int prism_b200_batch_create_tp(prism_b200_model *m, uint32_t sequences, uint32_t context,
                               uint32_t tp_rank, uint32_t tp_size, uint32_t tp_mode,
                               prism_b200_batch **out);
int prism_b200_batch_exchange_handle(const prism_b200_batch *b, void *handle);
int prism_b200_batch_connect(prism_b200_batch *b, const void *handles);
/* The slice rank `tp_rank` of `tp_size` owns (host only, no device):
 * out[0..12) = [first, end) of the query heads, the KV heads they read, the
 * Gated DeltaNet heads, the FFN intermediate's 256-row blocks, the output
 * head's vocabulary rows and the hidden rows of attn_output / ssm_out /
 * ffn_down in the exact form.  PRISM_B200_E_UNSUPPORTED when the
 * geometry does not split `tp_size` ways. */
int prism_b200_tp_plan(const prism_b200_qwen35_config *cfg, uint32_t tp_rank, uint32_t tp_size,
                       int32_t *out);

/* ---- synthetic inputs ----------------------------------------------- */
/* Fill `out` (host, rows*cols/256 blocks in the reference byte layout) with
 * seeded random packed weights: TQ2_0 codes uniform in {-1, 0, +1}, Q2_K
 * quants uniform in 0..3 with random 4-bit scales/mins; fp16 block scales
 * uniform in [scale_lo, scale_hi] (Q2_K dmin in half that range).  No
 * counterpart in the reference: it stands in for model files, which this
 * benchmark does not use.  Deterministic in (seed, stream). */
int prism_b200_synth_weights(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t seed,
                             uint64_t stream, float scale_lo, float scale_hi, void *out);

/* ---- weight inspection ---------------------------------------------- */
uint32_t prism_b200_weight_kind(const prism_b200_weight *w);
uint64_t prism_b200_weight_rows(const prism_b200_weight *w);
uint64_t prism_b200_weight_cols(const prism_b200_weight *w);
/* Bytes the weight occupies in HBM (equal to its packed byte size plus the
 * zero padding of the last 32-row tile). */
uint64_t prism_b200_weight_device_bytes(const prism_b200_weight *w);

/* Measured dense int8 tensor-core rate of the executor's device, in
 * Tint-op/s (2 per multiply-add): one CTA per SM issues `iters` back-to-back
 * tcgen05.mma.kind::i8 of 128x256x32 from shared memory.  No reference
 * counterpart; the denominator of the prefill GEMM's tensor roofline. */
int prism_b200_tensor_peak_i8(prism_b200_executor *ex, int iters, double *tops);

/* ---- rotated scalar KV codec ("rsq") --------------------------------- */
/* The reference's packed KV codec (reference src/kv_quant.rs `Quantizer`,
 * src/kv_quant/scalar.rs, fitted_scale.rs, tables.rs) for 256-channel rows:
 * a record is the binary32 scale |x|_2 / 16 (version 2: fitted to the codes)
 * then 256 codes of `bits` (3 or 4) bits, packed little-endian, of the row
 * normalised and rotated by three seeded sign flips and normalised
 * Walsh-Hadamard transforms; 100 or 132 bytes.  The policies use the fixed
 * seeds below (reference src/graph/quantized_kv.rs:80-84). */
#define PRISM_B200_KVQ_KEY_SEED 0x53574946544b5631ull
#define PRISM_B200_KVQ_VALUE_SEED 0x5357494654565631ull

/* Record bytes of a codec precision: 100 (3 bits), 132 (4 bits), else 0. */
int prism_b200_kvq_record_bytes(uint32_t bits);

/* Quantizer::encode of n rows (reference src/kv_quant.rs:515-565): rows
 * [n][256] binary32, records [n][record bytes].  version 1, or 2 for the
 * fitted scale (Quantizer::with_fitted_scale).  A nonfinite input or a
 * nonzero row whose scale underflows returns E_INVALID, an overflow
 * E_NONFINITE (the device-side status rules above). */
int prism_b200_kvq_encode(prism_b200_executor *ex, uint32_t bits, uint64_t seed,
                          uint32_t version, const float *rows, size_t n, uint8_t *records);
int prism_b200_kvq_encode_device(prism_b200_executor *ex, uint32_t bits, uint64_t seed,
                                 uint32_t version, const float *rows, size_t n,
                                 uint8_t *records, void *stream);

/* Quantizer::decode of n records (reference src/kv_quant.rs:812-822):
 * the reconstruction in the rotated basis, then the inverse rotation.  A
 * malformed record (negative, -0 or nonfinite scale; nonzero codes with a
 * zero scale) returns E_INVALID. */
int prism_b200_kvq_decode(prism_b200_executor *ex, uint32_t bits, uint64_t seed,
                          const uint8_t *records, size_t n, float *rows);

/* Gated attention of `heads` query heads over `positions` records
 * (reference src/graph/quantized_kv.rs:1302-1348 attend_head, Source
 * arithmetic), head h reading KV head h / (heads / kv_heads): the query row
 * rotated by the key codec, scores in four binary64 lanes times the record
 * scale times attn_scale, softmax_round_f16 over the positions in order,
 * the binary32 value scan in the rotated basis, the inverse value rotation,
 * then times sigmoid(gate).  queries, gates, out: [heads][256] binary32;
 * keys [positions][kv_heads][132], values [positions][kv_heads][132 | 100]
 * for `policy` PRISM_B200_KV_RSQ4, _RSQ4VF or _RSQ4K3V.  1..32768
 * positions. */
int prism_b200_kvq_attend(prism_b200_executor *ex, uint32_t policy, const float *queries,
                          const uint8_t *keys, const uint8_t *values, size_t positions,
                          uint32_t heads, uint32_t kv_heads, float attn_scale, const float *gates,
                          float *out);
int prism_b200_kvq_attend_device(prism_b200_executor *ex, uint32_t policy, const float *queries,
                                 const uint8_t *keys, const uint8_t *values, size_t positions,
                                 uint32_t heads, uint32_t kv_heads, float attn_scale,
                                 const float *gates, float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PRISM_B200_H */
