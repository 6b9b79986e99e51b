/*
 * prism_oracle.c -- CPU restatement of the prism-inference reference's
 * quantized-projection arithmetic (Source contract).
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the B200 kernels and the
 * timed CPU baseline of bench.py.  Nothing in the product library links,
 * loads or calls this code.
 *
 * Compile with -ffp-contract=off: every multiply and add below is a separate
 * binary32 (or binary64) rounding, exactly as the reference's Rust source
 * (which never contracts) performs them.
 *
 * Transcendentals: the reference calls f32::exp/ln/sin/cos, whose last-ulp
 * results depend on the host libm (glibc on Linux, the UCRT on Windows).
 * This restatement defines them as the correctly rounded binary32 value,
 * evaluated in binary64 and rounded once (po_expf etc.); the device kernels
 * use the same definition, so the two agree bit for bit.  A platform libm
 * differs from it only in rare last-ulp cases.
 */
#include "prism_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ---------------------------------------------------------------------- */
/* binary16 conversions                                                    */
/* ---------------------------------------------------------------------- */

/* Exact binary16 -> binary32 widening, preserving zero signs and NaN
 * payloads (reference tools/ternary/src/lib.rs:66-88, half_to_float). */
float po_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 31u;
  uint32_t man = h & 1023u;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    /* subnormal: value = man * 2^-24, renormalise */
    int e = -14;
    while (!(man & 1024u)) {
      man <<= 1;
      e -= 1;
    }
    man &= 1023u;
    return u2f(sign | ((uint32_t)(e + 127) << 23) | (man << 13));
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112u) << 23) | (man << 13));
}

/* binary32 -> binary16 with round-to-nearest-even, signed zero, subnormals
 * and infinities; every NaN becomes the quiet 0x7e00 with its sign
 * (the reference's float_to_half contract, tools/ternary/src/lib.rs:90-113).
 * Written from the IEEE 754 definition of the rounding. */
uint16_t po_float_to_half(float f) {
  uint32_t x = f2u(f);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return sign | 0x7e00u;      /* NaN */
  if (ax >= 0x477ff000u) return sign | 0x7c00u;     /* rounds to +-inf */
  if (ax >= 0x38800000u) {                          /* normal result */
    uint32_t h = ((((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13));
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return sign | (uint16_t)h;
  }
  if (ax <= 0x33000000u) return sign;               /* <= 2^-25 -> zero */
  /* subnormal result: round(value / 2^-24) */
  uint32_t e = ax >> 23;                            /* 102..112 here */
  uint32_t m = (ax & 0x7fffffu) | 0x800000u;        /* value = m * 2^(e-150) */
  uint32_t s = 126u - e;                            /* 14..24 */
  uint32_t h = m >> s;
  uint32_t rem = m & ((1u << s) - 1u);
  uint32_t half = 1u << (s - 1u);
  if (rem > half || (rem == half && (h & 1u))) h += 1u;
  return sign | (uint16_t)h;
}

float po_round_f16(float f) { return po_half_to_float(po_float_to_half(f)); }

static inline int finitef_(float v) { return isfinite(v) != 0; }

/* reference src/kernels.rs:152-154 `scale`: fp16 little-endian, must be finite */
static inline int read_scale(const uint8_t *p, float *out) {
  uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
  float v = po_half_to_float(h);
  if (!finitef_(v)) return PO_E_NONFINITE;
  *out = v;
  return PO_OK;
}

/* ---------------------------------------------------------------------- */
/* Q8_K / Q8_0 activation quantizers                                       */
/* ---------------------------------------------------------------------- */

/* reference src/kernels.rs:463-522 q8k_with_input (Source when !pinned);
 * pinned integer rounding follows src/kernels.rs:421-428. */
int po_q8k_quantize(const float *x, size_t n, int pinned, po_q8k_block *out) {
  if (n % 256 != 0) return PO_E_INVALID;
  size_t nb = n / 256;
  for (size_t b = 0; b < nb; ++b) {
    const float *c = x + b * 256;
    po_q8k_block *blk = out + b;
    float maximum = 0.0f;
    for (int i = 0; i < 256; ++i) {
      if (!finitef_(c[i])) goto fail_nonfinite;
      if (fabsf(c[i]) > fabsf(maximum)) maximum = c[i];
    }
    memset(blk, 0, sizeof(*blk));
    if (maximum == 0.0f) continue;
    float iscale = -127.0f / maximum;
    if (!finitef_(iscale)) goto fail_invalid;
    blk->scale = 1.0f / iscale;
    for (int i = 0; i < 256; ++i) {
      int q;
      if (pinned) {
        float r = fmaf(iscale, c[i], 12582912.0f);
        if (!finitef_(r)) goto fail_nonfinite;
        int32_t integer = (int32_t)(f2u(r) & 0x007fffffu) - 0x00400000;
        if (integer > 127) integer = 127;
        if (integer < -128) goto fail_invalid;
        q = integer;
      } else {
        float p = c[i] * iscale;
        float r = rintf(p);
        if (r > 127.0f) r = 127.0f;
        if (!(r >= -127.0f && r <= 127.0f)) goto fail_invalid;
        q = (int)r;
      }
      blk->values[i] = (int8_t)q;
    }
    for (int g = 0; g < 16; ++g) {
      int s = 0;
      for (int i = 0; i < 16; ++i) s += blk->values[g * 16 + i];
      blk->sums[g] = (int16_t)s;
    }
  }
  return PO_OK;
fail_nonfinite:
  memset(out, 0, nb * sizeof(*out));
  return PO_E_NONFINITE;
fail_invalid:
  memset(out, 0, nb * sizeof(*out));
  return PO_E_INVALID;
}

/* reference src/kernels.rs:552-617 q8_with_input<false,false,_>: d =
 * max|x|/127 stored as binary16, codes = round-half-away(x * (1/d)). */
int po_q8_0_quantize(const float *x, size_t n, po_q8_0_block *out) {
  if (n % 32 != 0) return PO_E_INVALID;
  size_t nb = n / 32;
  for (size_t b = 0; b < nb; ++b) {
    const float *c = x + b * 32;
    float maximum = 0.0f;
    for (int i = 0; i < 32; ++i) {
      if (!finitef_(c[i])) goto fail;
      maximum = fmaxf(maximum, fabsf(c[i]));
    }
    float d = maximum / 127.0f;
    float inverse = d == 0.0f ? 0.0f : 1.0f / d;
    uint16_t hb = po_float_to_half(d);
    if (!finitef_(po_half_to_float(hb))) goto fail;
    out[b].d = hb;
    for (int i = 0; i < 32; ++i) {
      float r = roundf(c[i] * inverse);
      if (!(r >= -127.0f && r <= 127.0f)) goto fail;
      out[b].values[i] = (int8_t)(int)r;
    }
  }
  return PO_OK;
fail:
  memset(out, 0, nb * sizeof(*out));
  return PO_E_NONFINITE;
}

/* ---------------------------------------------------------------------- */
/* TQ2_0                                                                   */
/* ---------------------------------------------------------------------- */

/* Element i of a TQ2_0 block sits in byte (i/128)*32 + i%32 at bit shift
 * 2*((i%128)/32); its weight is code-1 (so code 3 decodes to +2).
 * reference src/kernels/tquants.rs:45-57,148-167. */
static inline int tq2_code(const uint8_t *blk, int i) {
  return (int)((blk[(i / 128) * 32 + (i % 32)] >> (2 * ((i % 128) / 32))) & 3) - 1;
}

/* reference src/kernels/tquants.rs:258-268 decode */
int po_tq2_decode(const uint8_t *blocks, size_t nblocks, float *out) {
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 66;
    float d;
    if (read_scale(blk + 64, &d)) return PO_E_NONFINITE;
    for (int i = 0; i < 256; ++i) {
      float v = (float)tq2_code(blk, i) * d;
      if (!finitef_(v)) return PO_E_NONFINITE;
      out[b * 256 + i] = v;
    }
  }
  return PO_OK;
}

/* reference src/kernels/tquants.rs:288-336 quantize (kind 35) */
int po_tq2_quantize(const float *x, size_t n, uint8_t *out) {
  if (n == 0 || n % 256 != 0) return PO_E_INVALID;
  for (size_t i = 0; i < n; ++i)
    if (!finitef_(x[i])) return PO_E_INVALID;
  size_t nb = n / 256;
  memset(out, 0, nb * 66);
  for (size_t b = 0; b < nb; ++b) {
    const float *c = x + b * 256;
    uint8_t *o = out + b * 66;
    float d = 0.0f;
    for (int i = 0; i < 256; ++i) d = fmaxf(d, fabsf(c[i]));
    uint16_t bits = po_float_to_half(d);
    if (!finitef_(po_half_to_float(bits))) return PO_E_NONFINITE;
    o[64] = (uint8_t)(bits & 0xff);
    o[65] = (uint8_t)(bits >> 8);
    float inverse = 0.0f;
    if (d != 0.0f) {
      inverse = 1.0f / d;
      if (!finitef_(inverse)) return PO_E_NONFINITE;
    }
    for (int i = 0; i < 256; ++i) {
      int level = (int)(int16_t)roundf(c[i] * inverse) + 1;
      o[(i / 128) * 32 + (i % 32)] |= (uint8_t)((uint8_t)level << (2 * ((i % 128) / 32)));
    }
  }
  return PO_OK;
}

/* Signed digits (code-1) of the four 2-bit fields of every byte value
 * (reference src/kernels/tquants.rs:45-57 TQ2_BYTE_LUT). */
static int8_t g_tq2_lut[256][4];
static pthread_once_t g_tq2_once = PTHREAD_ONCE_INIT;
static void tq2_lut_init(void) {
  for (int b = 0; b < 256; ++b)
    for (int j = 0; j < 4; ++j) g_tq2_lut[b][j] = (int8_t)(((b >> (2 * j)) & 3) - 1);
}

/* reference src/kernels/tquants.rs:220-245 dot_tq2_block: exact i32 sum of
 * (code-1)*q over the block's 256 elements, one lookup per packed byte. */
static inline int32_t tq2_block_int(const uint8_t *blk, const int8_t *q) {
  pthread_once(&g_tq2_once, tq2_lut_init);
  int32_t sum = 0;
  for (int half = 0; half < 2; ++half) {
    const uint8_t *bytes = blk + half * 32;
    const int8_t *v = q + half * 128;
    for (int col = 0; col < 32; ++col) {
      const int8_t *d = g_tq2_lut[bytes[col]];
      sum += d[0] * (int32_t)v[col] + d[1] * (int32_t)v[col + 32] +
             d[2] * (int32_t)v[col + 64] + d[3] * (int32_t)v[col + 96];
    }
  }
  return sum;
}

int po_tq2_block_dots(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
                      int32_t *ints) {
  for (size_t b = 0; b < nblocks; ++b) ints[b] = tq2_block_int(w + b * 66, a[b].values);
  return PO_OK;
}

/* reference src/kernels/tquants.rs:270-287 dot: sum += (f32)int * (d * s),
 * binary32, sequential over blocks, then a finiteness check. */
int po_tq2_dot(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
               float *out) {
  float sum = 0.0f;
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = w + b * 66;
    int32_t integer = tq2_block_int(blk, a[b].values);
    float d;
    if (read_scale(blk + 64, &d)) return PO_E_NONFINITE;
    if (!finitef_(a[b].scale)) return PO_E_NONFINITE;
    float ds = d * a[b].scale;
    float term = (float)integer * ds;
    sum = sum + term;
  }
  if (!finitef_(sum)) return PO_E_NONFINITE;
  *out = sum;
  return PO_OK;
}

/* ---------------------------------------------------------------------- */
/* Q2_K                                                                    */
/* ---------------------------------------------------------------------- */

/* Q2_K block: scales[16] (low nibble scale, high nibble min) at 0..15,
 * 2-bit quants at 16..79 laid out like TQ2_0, fp16 d at 80, fp16 dmin at
 * 82.  reference src/kernels/kquants.rs:53-79. */
static inline int q2k_q(const uint8_t *blk, int i) {
  return (blk[16 + (i / 128) * 32 + (i % 32)] >> (2 * ((i % 128) / 32))) & 3;
}

/* reference src/kernels/kquants.rs:146-160 decode (kind 10) */
int po_q2k_decode(const uint8_t *blocks, size_t nblocks, float *out) {
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 84;
    float d, mn;
    if (read_scale(blk + 80, &d)) return PO_E_NONFINITE;
    if (read_scale(blk + 82, &mn)) return PO_E_NONFINITE;
    for (int i = 0; i < 256; ++i) {
      int g = i / 16;
      float sc = (float)(blk[g] & 15);
      float m = (float)(blk[g] >> 4);
      float t = (d * sc) * (float)q2k_q(blk, i);
      float v = t - mn * m;
      if (!finitef_(v)) return PO_E_NONFINITE;
      out[b * 256 + i] = v;
    }
  }
  return PO_OK;
}

/* reference src/kernels/kquants.rs:162-200 dot_q2_k_block, integer part:
 * isum = sum_g sc_g * sum_{i in g} q_i a_i ; msum = sum_g sums_g * min_g
 * (the activation block's stored group sums, as given). */
static inline void q2k_block_ints(const uint8_t *blk, const po_q8k_block *a,
                                  int32_t *isum, int32_t *msum) {
  int32_t is = 0, ms = 0;
  for (int g = 0; g < 16; ++g) {
    int32_t sub = 0;
    for (int i = g * 16; i < g * 16 + 16; ++i) sub += q2k_q(blk, i) * (int32_t)a->values[i];
    is += (int32_t)(blk[g] & 15) * sub;
    ms += (int32_t)a->sums[g] * (int32_t)(blk[g] >> 4);
  }
  *isum = is;
  *msum = ms;
}

int po_q2k_block_dots(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
                      int32_t *isum, int32_t *msum) {
  for (size_t b = 0; b < nblocks; ++b) q2k_block_ints(w + b * 84, a + b, isum + b, msum + b);
  return PO_OK;
}

/* reference src/kernels/kquants.rs:346-420 dot (kind 10):
 * sum += (s*d)*(f32)isum - (s*dmin)*(f32)msum, binary32, sequential. */
int po_q2k_dot(const uint8_t *w, const po_q8k_block *a, size_t nblocks,
               float *out) {
  float sum = 0.0f;
  for (size_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = w + b * 84;
    float s = a[b].scale;
    if (!finitef_(s)) return PO_E_NONFINITE;
    float d, mn;
    if (read_scale(blk + 80, &d)) return PO_E_NONFINITE;
    if (read_scale(blk + 82, &mn)) return PO_E_NONFINITE;
    int32_t is, ms;
    q2k_block_ints(blk, a + b, &is, &ms);
    float sd = s * d;
    float t1 = sd * (float)is;
    float sm = s * mn;
    float t2 = sm * (float)ms;
    float term = t1 - t2;
    sum = sum + term;
  }
  if (!finitef_(sum)) return PO_E_NONFINITE;
  *out = sum;
  return PO_OK;
}

/* ---------------------------------------------------------------------- */
/* Row-parallel matvec                                                     */
/* ---------------------------------------------------------------------- */

int po_block_bytes(uint32_t kind) {
  if (kind == 35) return 66;
  if (kind == 10) return 84;
  return po_ext_block_bytes(kind);  /* 34, 11-14 */
}

static int po_row_dot(uint32_t kind, const uint8_t *row, const po_q8k_block *a, size_t nb,
                      float *y) {
  if (kind == 35) return po_tq2_dot(row, a, nb, y);
  if (kind == 10) return po_q2k_dot(row, a, nb, y);
  return po_ext_dot(kind, row, a, nb, y);
}

typedef struct {
  uint32_t kind;
  const uint8_t *w;
  size_t row_begin, row_end, nb;
  const po_q8k_block *a;
  float *y;
  size_t first_error_row;
  int first_error;
} po_chunk;

static void *po_chunk_run(void *arg) {
  po_chunk *c = (po_chunk *)arg;
  size_t rb = (size_t)po_block_bytes(c->kind) * c->nb;
  c->first_error = PO_OK;
  for (size_t r = c->row_begin; r < c->row_end; ++r) {
    const uint8_t *row = c->w + r * rb;
    int st = po_row_dot(c->kind, row, c->a, c->nb, c->y + r);
    if (st != PO_OK) {
      c->first_error = st;
      c->first_error_row = r;
      return NULL;
    }
  }
  return NULL;
}

/* Contiguous output-row chunks of rows.div_ceil(workers), at most one task
 * per worker, the first error in row order reported
 * (reference src/kernels/parallel_rows.rs:507-542,602-628). */
int po_matvec(uint32_t kind, const uint8_t *w, size_t rows, size_t cols,
              const po_q8k_block *a, float *y, int threads) {
  if (po_block_bytes(kind) == 0 || cols == 0 || cols % 256 != 0 || rows == 0)
    return PO_E_INVALID;
  size_t nb = cols / 256;
  if (threads < 1) threads = 1;
  if ((size_t)threads > rows) threads = (int)rows;
  size_t chunk = (rows + (size_t)threads - 1) / (size_t)threads;
  int workers = (int)((rows + chunk - 1) / chunk);
  po_chunk *cs = (po_chunk *)calloc((size_t)workers, sizeof(po_chunk));
  pthread_t *ts = (pthread_t *)calloc((size_t)workers, sizeof(pthread_t));
  if (!cs || !ts) {
    free(cs);
    free(ts);
    return PO_E_INVALID;
  }
  for (int i = 0; i < workers; ++i) {
    cs[i].kind = kind;
    cs[i].w = w;
    cs[i].row_begin = (size_t)i * chunk;
    cs[i].row_end = cs[i].row_begin + chunk < rows ? cs[i].row_begin + chunk : rows;
    cs[i].nb = nb;
    cs[i].a = a;
    cs[i].y = y;
  }
  for (int i = 1; i < workers; ++i) pthread_create(&ts[i], NULL, po_chunk_run, &cs[i]);
  po_chunk_run(&cs[0]);
  for (int i = 1; i < workers; ++i) pthread_join(ts[i], NULL);
  int st = PO_OK;
  for (int i = 0; i < workers; ++i)
    if (cs[i].first_error != PO_OK) {
      st = cs[i].first_error;
      break;
    }
  free(cs);
  free(ts);
  if (st != PO_OK) memset(y, 0, rows * sizeof(float));
  return st;
}

/* Multi-token projection: the reference's tiled prefill shares each weight
 * row across a tile of at most 32 tokens and computes one per-token dot for
 * each (src/kernels/prefill.rs:26 MAX_TILE_TOKENS, :48-87
 * dot_quantized_tile_row); tokens are quantized to Q8_K once up front. */
#define PO_TILE_TOKENS 32

typedef struct {
  uint32_t kind;
  const uint8_t *w;
  size_t row_begin, row_end, nb, rows, tokens;
  const po_q8k_block *a; /* [tokens][nb] */
  float *y;              /* [tokens][rows] */
  int first_error;
} po_tile_chunk;

static void *po_tile_chunk_run(void *arg) {
  po_tile_chunk *c = (po_tile_chunk *)arg;
  size_t rb = (size_t)po_block_bytes(c->kind) * c->nb;
  c->first_error = PO_OK;
  for (size_t t0 = 0; t0 < c->tokens; t0 += PO_TILE_TOKENS) {
    size_t t1 = t0 + PO_TILE_TOKENS < c->tokens ? t0 + PO_TILE_TOKENS : c->tokens;
    for (size_t r = c->row_begin; r < c->row_end; ++r) {
      const uint8_t *row = c->w + r * rb;
      for (size_t t = t0; t < t1; ++t) {
        const po_q8k_block *a = c->a + t * c->nb;
        float *out = c->y + t * c->rows + r;
        int st = po_row_dot(c->kind, row, a, c->nb, out);
        if (st != PO_OK) {
          c->first_error = st;
          return NULL;
        }
      }
    }
  }
  return NULL;
}

int po_project_tokens(uint32_t kind, const uint8_t *w, size_t rows, size_t cols,
                      const float *x, size_t tokens, int pinned, float *y, int threads) {
  if (po_block_bytes(kind) == 0 || cols == 0 || cols % 256 != 0 || rows == 0)
    return PO_E_INVALID;
  if (tokens == 0) return PO_OK;
  size_t nb = cols / 256;
  po_q8k_block *a = (po_q8k_block *)malloc(tokens * nb * sizeof(po_q8k_block));
  if (!a) return PO_E_INVALID;
  int st = PO_OK;
  for (size_t t = 0; t < tokens && st == PO_OK; ++t)
    st = po_q8k_quantize(x + t * cols, cols, pinned, a + t * nb);
  if (st != PO_OK) {
    free(a);
    memset(y, 0, tokens * rows * sizeof(float));
    return st;
  }
  if (threads < 1) threads = 1;
  if ((size_t)threads > rows) threads = (int)rows;
  size_t chunk = (rows + (size_t)threads - 1) / (size_t)threads;
  int workers = (int)((rows + chunk - 1) / chunk);
  po_tile_chunk *cs = (po_tile_chunk *)calloc((size_t)workers, sizeof(po_tile_chunk));
  pthread_t *ts = (pthread_t *)calloc((size_t)workers, sizeof(pthread_t));
  if (!cs || !ts) {
    free(cs);
    free(ts);
    free(a);
    return PO_E_INVALID;
  }
  for (int i = 0; i < workers; ++i) {
    cs[i].kind = kind;
    cs[i].w = w;
    cs[i].row_begin = (size_t)i * chunk;
    cs[i].row_end = cs[i].row_begin + chunk < rows ? cs[i].row_begin + chunk : rows;
    cs[i].nb = nb;
    cs[i].rows = rows;
    cs[i].tokens = tokens;
    cs[i].a = a;
    cs[i].y = y;
  }
  for (int i = 1; i < workers; ++i) pthread_create(&ts[i], NULL, po_tile_chunk_run, &cs[i]);
  po_tile_chunk_run(&cs[0]);
  for (int i = 1; i < workers; ++i) pthread_join(ts[i], NULL);
  for (int i = 0; i < workers; ++i)
    if (cs[i].first_error != PO_OK) {
      st = cs[i].first_error;
      break;
    }
  free(cs);
  free(ts);
  free(a);
  if (st != PO_OK) memset(y, 0, tokens * rows * sizeof(float));
  return st;
}

/* ---------------------------------------------------------------------- */
/* Float primitives (Source contract)                                      */
/* ---------------------------------------------------------------------- */

/* reference src/kernels.rs:1256-1273 float_dot: binary32 products summed in
 * binary64 (from the iterator sum's -0.0 identity), rounded to binary32. */
float po_float_dot(const float *a, const float *b, size_t n) {
  double acc = -0.0;
  for (size_t i = 0; i < n; ++i) {
    float p = a[i] * b[i];
    acc += (double)p;
  }
  return (float)acc;
}

/* reference src/kernels.rs:1344-1360 f16_dot */
float po_f16_dot(const float *a, const uint16_t *b, size_t n) {
  double acc = -0.0;
  for (size_t i = 0; i < n; ++i) {
    float p = a[i] * po_half_to_float(b[i]);
    acc += (double)p;
  }
  return (float)acc;
}

/* Correctly rounded binary32 transcendentals (see the file header). */
float po_expf(float x) { return (float)exp((double)x); }
float po_logf(float x) { return (float)log((double)x); }
float po_sinf(float x) { return (float)sin((double)x); }
float po_cosf(float x) { return (float)cos((double)x); }

/* reference src/kernels.rs:3365-3368 */
float po_silu(float v) { return v / (1.0f + po_expf(-v)); }

/* reference src/graph.rs:6349-6351 */
float po_sigmoid(float v) { return 1.0f / (1.0f + po_expf(-v)); }

/* reference src/graph.rs:6357-6384 recurrent_decay */
int po_recurrent_decay(float alpha, float time_bias, float decay_weight,
                       float *out) {
  if (!finitef_(alpha) || !finitef_(time_bias) || !finitef_(decay_weight))
    return PO_E_NONFINITE;
  if (decay_weight > 0.0f) return PO_E_INVALID;
  if (decay_weight == 0.0f) {
    *out = 1.0f;
    return PO_OK;
  }
  float linear = alpha + time_bias;
  if (linear >= 88.0f) {
    if (!finitef_(linear)) {
      *out = 0.0f;
      return PO_OK;
    }
    *out = po_expf(linear * decay_weight);
    return PO_OK;
  }
  float softplus = linear > 20.0f ? linear : po_logf(1.0f + po_expf(linear));
  *out = po_expf(softplus * decay_weight);
  return PO_OK;
}

/* reference src/kernels.rs:3823-3878 rms_norm_scale_inner + 3388-3418 */
int po_rms_norm(const float *x, const float *w, size_t n, float eps,
                float *out) {
  if (n == 0 || !finitef_(eps) || eps < 0.0f) return PO_E_INVALID;
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) {
    if (!finitef_(x[i]) || !finitef_(w[i])) return PO_E_NONFINITE;
    float sq = x[i] * x[i];
    sum += (double)sq;
  }
  float mean = (float)(sum / (double)(uint32_t)n);
  float scale = 1.0f / sqrtf(mean + eps);
  if (!finitef_(scale) || scale <= 0.0f) return PO_E_INVALID;
  for (size_t i = 0; i < n; ++i) {
    float v = (x[i] * scale) * w[i];
    if (!finitef_(v)) return PO_E_NONFINITE;
    out[i] = v;
  }
  return PO_OK;
}

/* reference src/kernels.rs:3457-3488 add_rms_norm_into + 3904-3950:
 * values += delta (in place), then normalise the sum. */
int po_add_rms_norm(float *values, const float *delta, const float *w,
                    size_t n, float eps, float *out) {
  if (n == 0 || !finitef_(eps) || eps < 0.0f) return PO_E_INVALID;
  double sum = 0.0;
  int all_finite = 1;
  for (size_t i = 0; i < n; ++i) {
    float v = values[i] + delta[i];
    all_finite &= finitef_(v) && finitef_(w[i]);
    float sq = v * v;
    sum += (double)sq;
  }
  if (!all_finite) return PO_E_NONFINITE;
  float mean = (float)(sum / (double)(uint32_t)n);
  float scale = 1.0f / sqrtf(mean + eps);
  if (!finitef_(scale) || scale <= 0.0f) return PO_E_INVALID;
  for (size_t i = 0; i < n; ++i) values[i] = values[i] + delta[i];
  for (size_t i = 0; i < n; ++i) {
    float v = (values[i] * scale) * w[i];
    if (!finitef_(v)) return PO_E_NONFINITE;
    out[i] = v;
  }
  return PO_OK;
}

/* reference src/kernels.rs:3333-3352 l2_norm_in_place (ClampedL2) */
void po_l2_norm(float *x, size_t n, float eps) {
  double squares = -0.0;
  for (size_t i = 0; i < n; ++i) {
    float sq = x[i] * x[i];
    squares += (double)sq;
  }
  float scale = 1.0f / fmaxf(sqrtf((float)squares), eps);
  for (size_t i = 0; i < n; ++i) x[i] = x[i] * scale;
}

/* reference src/kernels.rs:4431-4466 softmax_round_f16 */
int po_softmax_round_f16(float *v, size_t n) {
  float maximum = -INFINITY;
  for (size_t i = 0; i < n; ++i) maximum = fmaxf(maximum, v[i]);
  if (!finitef_(maximum)) return PO_E_INVALID;
  for (size_t i = 0; i < n; ++i)
    if (isnan(v[i]) || v[i] == INFINITY) return PO_E_INVALID;
  double total = 0.0;
  for (size_t i = 0; i < n; ++i) {
    v[i] = po_expf(v[i] - maximum);
    total += (double)v[i];
  }
  float inverse = (float)(1.0 / total);
  for (size_t i = 0; i < n; ++i) v[i] = po_round_f16(v[i] * inverse);
  return PO_OK;
}
