/*
 * packed_oracle.c -- the reference's own packed ternary formats, PQ2 (type
 * 142) and PTQ1 (type 143), restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY: never linked into the product library.
 *
 * PQ2: 128 weights in 34 bytes, a binary16 scale then 32 bytes of 2-bit
 * codes, weight = code - 1 (code 3 decodes to +2, the native decoder's
 * value; reference src/kernels.rs:178-180).  PTQ1: the same 128 ternary
 * weights in 28 bytes, 26 bytes of base-3 fractional digits then the
 * binary16 scale (reference tools/ternary/src/lib.rs:193-250): each byte b
 * stands for the digits of b / 256 in base 3, five per byte for the first 24
 * bytes (weights 0-79 over bytes 0-15, 80-119 over bytes 16-23, digit d of
 * byte m the weight m + d * width), four for the last two (weights 120-127).
 *
 * Dots (reference src/kernels.rs:941-1060):
 *   - Q8_K activations (PQ2 with a multiple of 256 columns): per PQ2 block
 *     i, d = scale_i * act[i / 2].scale, s = the exact integer dot over the
 *     block's half of the activation block, output = output + d * s (or
 *     fma(d, s, output) when fused), blocks in order;
 *   - Q8_0 activations (PTQ1, and PQ2 otherwise): per block, s = sum over
 *     its four 32-weight groups of act.scale * dot (binary32, in order),
 *     output = output + d * s.
 * The build keeps every multiply and add separate (-ffp-contract=off).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "prism_oracle.h"

/* digits[b][d]: base-3 digit d of b / 256 (reference ptq_digits, tools/
 * ternary/src/lib.rs:203-229: multiply the fraction by 3, the integer part
 * is the digit). */
static uint8_t g_digits[256][5];
static int g_digits_ready = 0;

static void ptq_digits_init(void) {
  if (g_digits_ready) return;
  for (int b = 0; b < 256; ++b) {
    unsigned fraction = (unsigned)b;
    for (int d = 0; d < 5; ++d) {
      fraction *= 3u;
      g_digits[b][d] = (uint8_t)(fraction >> 8);
      fraction &= 255u;
    }
  }
  g_digits_ready = 1;
}

void po_pq2_values(const uint8_t *block, int16_t *out) {
  for (int i = 0; i < 128; ++i) out[i] = (int16_t)(((block[2 + i / 4] >> (2 * (i % 4))) & 3) - 1);
}

void po_ptq1_values(const uint8_t *block, int16_t *out) {
  ptq_digits_init();
  for (int i = 0; i < 128; ++i) {
    int lane, digit;
    if (i < 80) {
      lane = i % 16;
      digit = i / 16;
    } else if (i < 120) {
      lane = 16 + (i - 80) % 8;
      digit = (i - 80) / 8;
    } else {
      lane = 24 + (i - 120) % 2;
      digit = (i - 120) / 2;
    }
    out[i] = (int16_t)(g_digits[block[lane]][digit] - 1);
  }
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* The binary16 scale of a block (finite), as the reference's scale(). */
static int block_scale(uint32_t kind, const uint8_t *block, float *d) {
  const float s = po_half_to_float(rd16(kind == 142 ? block : block + 26));
  if (!isfinite(s)) return PO_E_NONFINITE;
  *d = s;
  return PO_OK;
}

int po_packed_block_bytes(uint32_t kind) {
  return kind == 142 ? 34 : kind == 143 ? 28 : 0;
}

static float integer_dot(const int16_t *w, const int8_t *a, int n) {
  int32_t s = 0;
  for (int i = 0; i < n; ++i) s += (int32_t)w[i] * (int32_t)a[i];
  return (float)s;
}

int po_pq2_dot_q8k(const uint8_t *w, size_t nblocks, const po_q8k_block *a, int fused,
                   float *out) {
  float output = 0.0f;
  int16_t v[128];
  for (size_t i = 0; i < nblocks; ++i) {
    const uint8_t *block = w + i * 34;
    float scale;
    const int st = block_scale(142, block, &scale);
    if (st) return st;
    const po_q8k_block *act = &a[i / 2];
    const float d = scale * act->scale;
    po_pq2_values(block, v);
    const float sum = integer_dot(v, act->values + (i % 2) * 128, 128);
    output = fused ? fmaf(d, sum, output) : output + d * sum;
  }
  if (!isfinite(output)) return PO_E_NONFINITE;
  *out = output;
  return PO_OK;
}

int po_packed_dot_q8(uint32_t kind, const uint8_t *w, size_t nblocks, const po_q8_0_block *a,
                     float *out) {
  const int bb = po_packed_block_bytes(kind);
  if (!bb) return PO_E_INVALID;
  float output = 0.0f;
  int16_t v[128];
  for (size_t i = 0; i < nblocks; ++i) {
    const uint8_t *block = w + i * (size_t)bb;
    float d;
    const int st = block_scale(kind, block, &d);
    if (st) return st;
    if (kind == 142)
      po_pq2_values(block, v);
    else
      po_ptq1_values(block, v);
    float sum = 0.0f;
    for (int g = 0; g < 4; ++g) {
      const po_q8_0_block *act = &a[i * 4 + g];
      sum += po_half_to_float(act->d) * integer_dot(v + 32 * g, act->values, 32);
    }
    output += d * sum;
  }
  if (!isfinite(output)) return PO_E_NONFINITE;
  *out = output;
  return PO_OK;
}

/* The activation contract (reference src/kernels.rs:1663-1674): PQ2 with a
 * multiple of 256 columns takes Q8_K, PQ2 otherwise and PTQ1 take Q8_0. */
int po_packed_uses_q8k(uint32_t kind, size_t cols) { return kind == 142 && cols % 256 == 0; }

int po_packed_matvec(uint32_t kind, const uint8_t *w, size_t rows, size_t cols, const float *x,
                     int fused, float *y) {
  const int bb = po_packed_block_bytes(kind);
  if (!bb || cols == 0 || cols % 128) return PO_E_INVALID;
  const size_t nb = cols / 128;
  int st = PO_OK;
  if (po_packed_uses_q8k(kind, cols)) {
    po_q8k_block *a = (po_q8k_block *)malloc(sizeof(po_q8k_block) * (cols / 256));
    if (!a) return PO_E_INVALID;
    st = po_q8k_quantize(x, cols, 0, a);
    for (size_t r = 0; r < rows && !st; ++r) st = po_pq2_dot_q8k(w + r * nb * 34, nb, a, fused, &y[r]);
    free(a);
  } else {
    po_q8_0_block *a = (po_q8_0_block *)malloc(sizeof(po_q8_0_block) * (cols / 32));
    if (!a) return PO_E_INVALID;
    st = po_q8_0_quantize(x, cols, a);
    for (size_t r = 0; r < rows && !st; ++r)
      st = po_packed_dot_q8(kind, w + r * nb * (size_t)bb, nb, a, &y[r]);
    free(a);
  }
  if (st) memset(y, 0, rows * sizeof(float));
  return st;
}

/* Decoded row r: scale * weight, as the reference's row(). */
int po_packed_row(uint32_t kind, const uint8_t *w, size_t cols, size_t r, float *out) {
  const int bb = po_packed_block_bytes(kind);
  if (!bb || cols % 128) return PO_E_INVALID;
  const size_t nb = cols / 128;
  int16_t v[128];
  for (size_t i = 0; i < nb; ++i) {
    const uint8_t *block = w + (r * nb + i) * (size_t)bb;
    float d;
    const int st = block_scale(kind, block, &d);
    if (st) return st;
    if (kind == 142)
      po_pq2_values(block, v);
    else
      po_ptq1_values(block, v);
    for (int j = 0; j < 128; ++j) out[i * 128 + j] = d * (float)v[j];
  }
  return PO_OK;
}
