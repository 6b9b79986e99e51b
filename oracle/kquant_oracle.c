/*
 * kquant_oracle.c -- the remaining kinds of the reference's Q8_K activation
 * contract (src/kernels.rs:1653-1674): TQ1_0 (34) and Q3_K, Q4_K, Q5_K, Q6_K
 * (11-14), restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY: never linked into the product library.
 *
 * Each kind has a decode (the block's weights as binary32) and a dot against
 * Q8_K activation blocks (binary32 arithmetic, every operation separately
 * rounded: the build uses -ffp-contract=off):
 *   - TQ1_0 (54 B): 48 bytes of five base-3 digits, 4 bytes of four, fp16 d;
 *     dot as TQ2_0's: sum += (f32)int * (d * s) per block
 *     (reference src/kernels/tquants.rs:148-188, 190-216, 270-287);
 *   - Q3_K (110 B), Q4_K (144 B), Q5_K (176 B), Q6_K (210 B): per block, the
 *     exact integer sums of 8 lanes (element j of a group goes to lane j % 8)
 *     weighted by the group scales; then lane[l] += (d * s) * (f32)int[l],
 *     blocks in order; Q4_K/Q5_K also sum -= (dmin * s) * (f32)msum per
 *     block; at the end sum += lane[0..7] in order
 *     (reference src/kernels/kquants.rs:53-130, 137-155, 202-420).
 */
#include <math.h>
#include <string.h>

#include "prism_oracle.h"

static int scale16(const uint8_t *p, float *out) {
  const float v = po_half_to_float((uint16_t)(p[0] | (p[1] << 8)));
  if (!isfinite(v)) return PO_E_NONFINITE;
  *out = v;
  return PO_OK;
}

int po_ext_block_bytes(uint32_t kind) {
  switch (kind) {
    case 34: return 54;
    case 11: return 110;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    default: return 0;
  }
}

/* TQ1_0 digit e (0..4) of byte b: the integer part of 3 * ((b * 3^e) mod 256)
 * / 256, minus one (reference src/kernels/tquants.rs:25-41 TQ1_BYTE_LUT). */
static int tq1_digit(uint8_t b, int e) {
  static const uint8_t pow3[5] = {1, 3, 9, 27, 81};
  const uint8_t m = (uint8_t)(b * pow3[e]);
  return (int)m * 3 / 256 - 1;
}

/* The 256 signed TQ1_0 codes in element order (src/kernels/tquants.rs:162-186). */
static void tq1_codes(const uint8_t *blk, int16_t *out) {
  for (int col = 0; col < 32; ++col)
    for (int e = 0; e < 5; ++e) out[col + 32 * e] = (int16_t)tq1_digit(blk[col], e);
  for (int col = 0; col < 16; ++col)
    for (int e = 0; e < 5; ++e) out[160 + col + 16 * e] = (int16_t)tq1_digit(blk[32 + col], e);
  for (int col = 0; col < 4; ++col)
    for (int e = 0; e < 4; ++e) out[240 + col + 4 * e] = (int16_t)tq1_digit(blk[48 + col], e);
}

/* Q4_K / Q5_K group scale and minimum (6 bits each) of group g from the 12
 * packed bytes (reference tools/ternary/src/lib.rs:127-136). */
static void q45_scale_min(int g, const uint8_t *s, int *sc, int *mn) {
  if (g < 4) {
    *sc = s[g] & 63;
    *mn = s[g + 4] & 63;
  } else {
    *sc = (s[g + 4] & 15) | ((s[g - 4] >> 6) << 4);
    *mn = (s[g + 4] >> 4) | ((s[g] >> 6) << 4);
  }
}

/* A K-quant block unpacked (reference src/kernels/kquants.rs:53-130):
 * integer values, group scales and minima, d, dmin and the group width. */
typedef struct {
  int16_t values[256];
  int16_t scales[16], minima[16];
  float d, dmin;
  int group;
} kblock;

static int kunpack(uint32_t kind, const uint8_t *b, kblock *k) {
  memset(k, 0, sizeof(*k));
  k->group = 16;
  int st;
  switch (kind) {
    case 11:
      if ((st = scale16(b + 108, &k->d))) return st;
      for (int g = 0; g < 16; ++g)
        k->scales[g] = (int16_t)((((b[96 + g % 8] >> (4 * (g / 8))) & 15) |
                                  (((b[104 + g % 4] >> (2 * (g / 4))) & 3) << 4)) -
                                 32);
      for (int i = 0; i < 256; ++i) {
        const int low = (b[32 + i / 128 * 32 + i % 32] >> (2 * (i % 128 / 32))) & 3;
        const int sub = (b[i % 32] & (1 << (i / 32))) ? 0 : 4;
        k->values[i] = (int16_t)(low - sub);
      }
      return PO_OK;
    case 12:
    case 13: {
      k->group = 32;
      if ((st = scale16(b, &k->d))) return st;
      if ((st = scale16(b + 2, &k->dmin))) return st;
      for (int g = 0; g < 8; ++g) {
        int sc, mn;
        q45_scale_min(g, b + 4, &sc, &mn);
        k->scales[g] = (int16_t)sc;
        k->minima[g] = (int16_t)mn;
      }
      const int off = kind == 12 ? 16 : 48;
      for (int i = 0; i < 256; ++i) {
        int v = (b[off + i / 64 * 32 + i % 32] >> (4 * (i % 64 / 32))) & 15;
        if (kind == 13 && (b[16 + i % 32] & (1 << (i / 32)))) v += 16;
        k->values[i] = (int16_t)v;
      }
      return PO_OK;
    }
    case 14:
      if ((st = scale16(b + 208, &k->d))) return st;
      for (int g = 0; g < 16; ++g) k->scales[g] = (int16_t)(int8_t)b[192 + g];
      for (int i = 0; i < 256; ++i) {
        const int part = i % 128 / 32;
        const int low = (b[i / 128 * 64 + part % 2 * 32 + i % 32] >> (4 * (part / 2))) & 15;
        const int high = (b[128 + i / 128 * 32 + i % 32] >> (2 * part)) & 3;
        k->values[i] = (int16_t)((low | (high << 4)) - 32);
      }
      return PO_OK;
    default:
      return PO_E_INVALID;
  }
}

int po_ext_decode(uint32_t kind, const uint8_t *blocks, size_t nblocks, float *out) {
  const int bb = po_ext_block_bytes(kind);
  if (!bb) return PO_E_INVALID;
  for (size_t n = 0; n < nblocks; ++n) {
    const uint8_t *b = blocks + n * (size_t)bb;
    float *o = out + n * 256;
    int st;
    if (kind == 34) {
      float d;
      if ((st = scale16(b + 52, &d))) return st;
      int16_t c[256];
      tq1_codes(b, c);
      for (int i = 0; i < 256; ++i) {
        o[i] = (float)c[i] * d;
        if (!isfinite(o[i])) return PO_E_NONFINITE;
      }
      continue;
    }
    kblock k;
    if ((st = kunpack(kind, b, &k))) return st;
    for (int i = 0; i < 256; ++i) {
      const int g = i / k.group;
      o[i] = (k.d * (float)k.scales[g]) * (float)k.values[i] - k.dmin * (float)k.minima[g];
      if (!isfinite(o[i])) return PO_E_NONFINITE;
    }
  }
  return PO_OK;
}

/* The exact integer parts of one block against one Q8_K block: the 8 lane
 * sums (kinds 11-14), the minimum sum (12, 13), or the single sum (34). */
static int ext_block_ints(uint32_t kind, const uint8_t *b, const po_q8k_block *a,
                          int32_t lanes[8], int32_t *msum, kblock *k) {
  memset(lanes, 0, 8 * sizeof(int32_t));
  *msum = 0;
  if (kind == 34) {
    int16_t c[256];
    tq1_codes(b, c);
    int32_t s = 0;
    for (int i = 0; i < 256; ++i) s += (int32_t)c[i] * (int32_t)a->values[i];
    lanes[0] = s;
    return PO_OK;
  }
  const int st = kunpack(kind, b, k);
  if (st) return st;
  const int ng = 256 / k->group;
  for (int g = 0; g < ng; ++g) {
    int32_t sub[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < k->group; ++j) {
      const int i = g * k->group + j;
      sub[j % 8] += (int32_t)k->values[i] * (int32_t)a->values[i];
    }
    for (int l = 0; l < 8; ++l) lanes[l] += (int32_t)k->scales[g] * sub[l];
    if (kind == 12 || kind == 13)
      *msum += ((int32_t)a->sums[2 * g] + (int32_t)a->sums[2 * g + 1]) * (int32_t)k->minima[g];
  }
  return PO_OK;
}

int po_ext_block_ints(uint32_t kind, const uint8_t *w, const po_q8k_block *a, size_t nblocks,
                      int32_t *lanes, int32_t *msum) {
  const int bb = po_ext_block_bytes(kind);
  if (!bb) return PO_E_INVALID;
  kblock k;
  for (size_t n = 0; n < nblocks; ++n) {
    const int st = ext_block_ints(kind, w + n * (size_t)bb, a + n, lanes + 8 * n, msum + n, &k);
    if (st) return st;
  }
  return PO_OK;
}

int po_ext_dot(uint32_t kind, const uint8_t *w, const po_q8k_block *a, size_t nblocks,
               float *out) {
  const int bb = po_ext_block_bytes(kind);
  if (!bb) return PO_E_INVALID;
  float sum = 0.0f, lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  kblock k;
  for (size_t n = 0; n < nblocks; ++n) {
    const uint8_t *b = w + n * (size_t)bb;
    const float s = a[n].scale;
    int32_t ints[8], msum;
    int st = ext_block_ints(kind, b, a + n, ints, &msum, &k);
    if (st) return st;
    if (kind == 34) {
      float d;
      if ((st = scale16(b + 52, &d))) return st;
      if (!isfinite(s)) return PO_E_NONFINITE;
      const float ds = d * s;
      sum = sum + (float)ints[0] * ds;
      continue;
    }
    if (!isfinite(s)) return PO_E_NONFINITE;
    const float dact = k.d * s;
    for (int l = 0; l < 8; ++l) lane[l] = lane[l] + dact * (float)ints[l];
    if (kind == 12 || kind == 13) {
      const float ms = k.dmin * s;
      sum = sum - ms * (float)msum;
    }
  }
  if (kind != 34)
    for (int l = 0; l < 8; ++l) sum = sum + lane[l];
  if (!isfinite(sum)) return PO_E_NONFINITE;
  *out = sum;
  return PO_OK;
}

/* reference src/kernels/tquants.rs:288-336 quantize, kinds 34 and 35:
 * d = max |x| stored as binary16, level = round(x * (1 / d)) + 1 (0 when d
 * is 0), then TQ2_0's 2-bit fields or TQ1_0's base-3 bytes
 * ceil(code * 256 / 243) (four-digit bytes scaled by 3 first). */
int po_tq_quantize(uint32_t kind, const float *x, size_t n, uint8_t *out) {
  const int size = kind == 35 ? 66 : kind == 34 ? 54 : 0;
  if (!size || n == 0 || n % 256) return PO_E_INVALID;
  for (size_t i = 0; i < n; ++i)
    if (!isfinite(x[i])) return PO_E_INVALID;
  memset(out, 0, n / 256 * (size_t)size);
  for (size_t b = 0; b < n / 256; ++b) {
    const float *c = x + b * 256;
    uint8_t *o = out + b * (size_t)size;
    float d = 0.0f;
    for (int i = 0; i < 256; ++i) d = fmaxf(d, fabsf(c[i]));
    const uint16_t bits = po_float_to_half(d);
    if (!isfinite(po_half_to_float(bits))) return PO_E_NONFINITE;
    o[size - 2] = (uint8_t)(bits & 0xff);
    o[size - 1] = (uint8_t)(bits >> 8);
    float inverse = 0.0f;
    if (d != 0.0f) {
      inverse = 1.0f / d;
      if (!isfinite(inverse)) return PO_E_NONFINITE;
    }
    uint8_t level[256];
    for (int i = 0; i < 256; ++i) level[i] = (uint8_t)((int)(int16_t)roundf(c[i] * inverse) + 1);
    if (kind == 35) {
      for (int i = 0; i < 256; ++i)
        o[i / 128 * 32 + i % 32] |= (uint8_t)(level[i] << (2 * (i % 128 / 32)));
      continue;
    }
    for (int byte = 0; byte < 52; ++byte) {
      int first, stride, count;
      if (byte < 32) {
        first = byte; stride = 32; count = 5;
      } else if (byte < 48) {
        first = 160 + byte - 32; stride = 16; count = 5;
      } else {
        first = 240 + byte - 48; stride = 4; count = 4;
      }
      unsigned code = 0;
      for (int k = 0; k < count; ++k) code = code * 3 + level[first + k * stride];
      if (count == 4) code *= 3;
      o[byte] = (uint8_t)((code * 256 + 242) / 243);
    }
  }
  return PO_OK;
}
