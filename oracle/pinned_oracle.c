/*
 * pinned_oracle.c -- the reference's pinned ("Swift") arithmetic variants of
 * the GDN row, attention dot, softmax and RoPE, restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY: never linked into the product library.
 *
 * The reference keeps two arithmetic contracts (src/graph.rs:3085-3110).
 * Synthetic models, and so every benchmark here, take `Source`; `PinnedSwift`
 * reproduces the native ggml CPU build's NEON reduction trees and fused
 * multiply-adds for two verified model artifacts.  The reference pins the
 * pinned variant with native captures (tests/fixtures/swift-gdn-parity.*,
 * swift-attention-{dot,softmax,rope}.json, swift-rope-inplace.*).  These
 * functions restate that variant so the captures can be checked here bit for
 * bit; the Source functions of prism_oracle.c / qwen35_oracle.c differ from
 * them only in summation order and in fusing, which the tests show on the
 * same captured inputs.  fmaf is the reference's f32::mul_add (one
 * rounding); the build keeps every other multiply and add separate
 * (-ffp-contract=off).
 */
#include <math.h>
#include <string.h>

#include "prism_oracle.h"

static inline uint32_t bits_of(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float of_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Four 4-lane registers (sums[r][l]) reduced as the NEON build does:
 * registers 0+2 and 1+3 first, then adjacent lane pairs (reference
 * src/kernels/pinned_gdn.rs:219-225). */
static inline float reduce_four_registers(float sums[4][4]) {
  float lanes[4];
  for (int l = 0; l < 4; ++l) lanes[l] = (sums[0][l] + sums[2][l]) + (sums[1][l] + sums[3][l]);
  return (lanes[0] + lanes[1]) + (lanes[2] + lanes[3]);
}

/* reference src/kernels/pinned_gdn.rs:205-230 dot_scalar: fused multiply-adds
 * into 16 lanes over the 16-aligned prefix, the register tree, then a
 * separately rounded tail. */
float po_pinned_gdn_dot(const float *a, const float *b, size_t n) {
  const size_t vec = n / 16 * 16;
  float sums[4][4];
  memset(sums, 0, sizeof(sums));
  for (size_t off = 0; off < vec; off += 16)
    for (int r = 0; r < 4; ++r)
      for (int l = 0; l < 4; ++l) {
        const size_t i = off + (size_t)r * 4 + (size_t)l;
        sums[r][l] = fmaf(a[i], b[i], sums[r][l]);
      }
  float result = reduce_four_registers(sums);
  for (size_t i = vec; i < n; ++i) result += a[i] * b[i];
  return result;
}

/* reference src/kernels/pinned_gdn.rs:975-985 scalar_add_scaled: fused over
 * the 16-aligned prefix, separately rounded after it. */
int po_pinned_gdn_add_scaled(float *target, const float *input, float scale, size_t n) {
  const size_t vec = n / 16 * 16;
  for (size_t i = 0; i < n; ++i) {
    target[i] = i < vec ? fmaf(scale, input[i], target[i]) : target[i] + scale * input[i];
    if (!isfinite(target[i])) return PO_E_NONFINITE;
  }
  return PO_OK;
}

/* Padded dot steps of the native 256-token cache rows (reference
 * src/kernels/pinned_attention.rs:49-55): at most 16 masked zero lanes are
 * visited; more cannot change a finite result. */
static size_t padded_steps(size_t logical) {
  const size_t padded = (logical + 255) / 256 * 256;
  const size_t padding = padded - logical;
  return logical + (padding < 16 ? padding : 16);
}

/* reference src/kernels/pinned_attention.rs:1015-1039 dot: fused
 * multiply-adds into sums[i % 16 / 4][i % 4] over the padded steps (masked
 * steps add 0 * 0), then the register tree. */
int po_pinned_attention_dot(const float *values, const float *weights, size_t n, float *out) {
  if (n == 0) return PO_E_INVALID;
  float sums[4][4];
  memset(sums, 0, sizeof(sums));
  const size_t steps = padded_steps(n);
  for (size_t i = 0; i < steps; ++i) {
    const float v = i < n ? values[i] : 0.0f, w = i < n ? weights[i] : 0.0f;
    float *s = &sums[i % 16 / 4][i % 4];
    *s = fmaf(v, w, *s);
  }
  const float r = reduce_four_registers(sums);
  if (!isfinite(r)) return PO_E_NONFINITE;
  *out = r;
  return PO_OK;
}

/* The native build's vectorized exponential, lane by lane (reference
 * src/kernels/pinned_activations.rs:22-53, which restates the pinned ggml
 * ggml_v_expf): a rounding-to-integer split by log2(e), a two-term Cody-Waite
 * reduction, a degree-5 polynomial in fused form, and exponent assembly with
 * the over- and underflow branches. */
float po_vector_exp(float value) {
  const float z = fmaf(value, of_bits(0x3fb8aa3bu), 12582912.0f);
  const float n = z - 12582912.0f;
  float r = fmaf(-n, of_bits(0x3f317200u), value);
  r = fmaf(-n, of_bits(0x35bfbe8eu), r);
  const uint32_t e = bits_of(z) << 23;
  const float k = of_bits(e + bits_of(1.0f));
  const float sq = r * r;
  const float inner = fmaf(fmaf(of_bits(0x3c072010u), r, of_bits(0x3d2b9f17u)), sq,
                           fmaf(of_bits(0x3e2aaf33u), r, of_bits(0x3efffedbu)));
  const float poly = fmaf(inner, sq, of_bits(0x3f7ffff6u) * r);
  if (fabsf(n) > 126.0f) {
    const uint32_t shift = n <= 0.0f ? 0x82000000u : 0u;
    const float s1 = of_bits(shift + 0x7f000000u);
    if (fabsf(n) > 192.0f) return s1 * s1;
    const float s2 = of_bits(e - shift);
    return fmaf(s2, poly, s2) * s1;
  }
  return fmaf(poly, k, k);
}

/* reference src/kernels/pinned_attention.rs:1131-1158 (scalar path of
 * softmax_with_rounding): the maximum, the vector exponential of every
 * score minus it, groups of four summed pairwise in binary32 and added to a
 * binary64 total, the reciprocal taken in binary64 and rounded once, the
 * probabilities scaled in binary32 (and rounded to binary16 when asked). */
int po_pinned_softmax(float *scores, size_t n, int round_f16) {
  if (n == 0) return PO_E_INVALID;
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(scores[i])) return PO_E_INVALID;
  float maximum = -INFINITY;
  for (size_t i = 0; i < n; ++i) maximum = fmaxf(maximum, scores[i]);
  double total = 0.0;
  for (size_t off = 0; off < n; off += 4) {
    float g[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (size_t l = 0; l < 4 && off + l < n; ++l) {
      scores[off + l] = po_vector_exp(scores[off + l] - maximum);
      g[l] = scores[off + l];
    }
    total += (double)((g[0] + g[1]) + (g[2] + g[3]));
  }
  const float inverse = (float)(1.0 / total);
  for (size_t i = 0; i < n; ++i) {
    const float s = scores[i] * inverse;
    scores[i] = round_f16 ? po_round_f16(s) : s;
  }
  return PO_OK;
}

/* reference src/kernels/pinned_attention.rs:1290-1339 rope_with_aliasing
 * (scalar path): each pair (i, i + rotary/2) of each head, fused; the
 * in-place form's first component is first*cos fused with -(second*sin),
 * the out-of-place form's is -second*sin fused with first*cos. */
int po_pinned_rope(float *x, size_t n, int head, int rotary, const float *cos_sin, int in_place) {
  if (head <= 0 || rotary <= 0 || rotary > head || n % (size_t)head) return PO_E_INVALID;
  const int half = rotary / 2;
  for (size_t h = 0; h < n; h += (size_t)head) {
    float *v = x + h;
    for (int i = 0; i < half; ++i) {
      const float c = cos_sin[2 * i], s = cos_sin[2 * i + 1];
      const float first = v[i], second = v[i + half];
      v[i] = in_place ? fmaf(first, c, -(second * s)) : fmaf(-second, s, first * c);
      v[i + half] = fmaf(second, c, first * s);
    }
  }
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(x[i])) return PO_E_NONFINITE;
  return PO_OK;
}

/* The Source RoPE of the same pairs (reference src/graph.rs:6439-6449):
 * separately rounded products and sums. */
int po_source_rope(float *x, size_t n, int head, int rotary, const float *cos_sin) {
  if (head <= 0 || rotary <= 0 || rotary > head || n % (size_t)head) return PO_E_INVALID;
  const int half = rotary / 2;
  for (size_t h = 0; h < n; h += (size_t)head) {
    float *v = x + h;
    for (int i = 0; i < half; ++i) {
      const float c = cos_sin[2 * i], s = cos_sin[2 * i + 1];
      const float first = v[i], second = v[i + half];
      v[i] = first * c - second * s;
      v[i + half] = first * s + second * c;
    }
  }
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(x[i])) return PO_E_NONFINITE;
  return PO_OK;
}

/* One GDN state row over one token in the pinned arithmetic (reference
 * src/kernels/pinned_gdn.rs:370-398 step_row_in_place: decay_and_dot
 * :236-258, the unfused delta, update_and_dot :310-336): the row scaled by
 * decay (separate multiplies), dot_k = the pinned dot with the key,
 * delta = (value - dot_k) * beta, the row += delta * key (fused over the
 * 16-aligned prefix), then the pinned dot with the query.  Returns
 * PO_E_NONFINITE where the reference returns its nonfinite error. */
static int pinned_step_row(float *row, const float *key, const float *query, float decay,
                           float value, float beta, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) row[i] *= decay;
  const float dot_k = po_pinned_gdn_dot(row, key, n);
  if (!isfinite(dot_k)) return PO_E_NONFINITE;
  const float delta = (value - dot_k) * beta;
  if (po_pinned_gdn_add_scaled(row, key, delta, n)) return PO_E_NONFINITE;
  const float dot_q = po_pinned_gdn_dot(row, query, n);
  if (!isfinite(dot_q)) return PO_E_NONFINITE;
  *out = dot_q;
  return PO_OK;
}

/* Every head of every sequence over `tokens` tokens in the pinned
 * arithmetic, in the device GDN layout: q, k [batch][tokens][key_heads][d],
 * v, out [batch][tokens][heads][d], decay, beta [batch][tokens][heads],
 * state [batch][heads][d rows][d]; head h reads key head h % key_heads;
 * out = dot_q * scale with scale = 1 / sqrt(d) (the reference's
 * step_row_tokens_from, :401-455, rows of a head in any order: each row is
 * independent).  The state of a row that fails is left partially updated, as
 * the reference's error leaves it. */
int po_pinned_gdn_prefill(float *state, const float *q, const float *k, const float *v,
                          const float *decay, const float *beta, int batch, int tokens, int heads,
                          int key_heads, int d, float *out) {
  if (batch <= 0 || tokens <= 0 || heads <= 0 || key_heads <= 0 || heads % key_heads || d <= 0)
    return PO_E_INVALID;
  const float scale = 1.0f / sqrtf((float)d);
  int status = PO_OK;
  for (int b = 0; b < batch; ++b)
    for (int h = 0; h < heads; ++h) {
      float *S = state + ((size_t)b * heads + h) * (size_t)d * d;
      const int kh = h % key_heads;
      for (int t = 0; t < tokens; ++t) {
        const size_t tok = (size_t)b * tokens + t;
        const float *kk = k + (tok * key_heads + kh) * d, *qq = q + (tok * key_heads + kh) * d;
        const float *vv = v + (tok * heads + h) * d;
        const float g = decay[tok * heads + h], bt = beta[tok * heads + h];
        for (int r = 0; r < d; ++r) {
          float o = 0.0f;
          const int st = pinned_step_row(S + (size_t)r * d, kk, qq, g, vv[r], bt, (size_t)d, &o);
          if (st && !status) status = st;
          out[(tok * heads + h) * d + r] = o * scale;
        }
      }
    }
  return status;
}
