/*
 * kvq_oracle.c -- the reference's rotated scalar KV codec (src/kv_quant.rs,
 * "rsq") and the attention over its records (src/graph/quantized_kv.rs),
 * restated on the CPU.
 *
 * TEST INFRASTRUCTURE ONLY: never linked into the product library.
 *
 * A 256-channel row is normalised by scale = |row|_2 / 16 (binary64 FMA
 * chain in channel order, binary32 result), rotated by three passes of a
 * seeded sign flip followed by the normalised Walsh-Hadamard transform, and
 * each rotated coordinate is coded as its nearest symmetric Gaussian
 * Lloyd-Max level (8 or 16 levels; the first-code tie rule).  A record is the
 * binary32 scale then the codes packed little-endian, 3 or 4 bits each (100
 * or 132 bytes).  Version 2 fits the stored scale to the chosen codes.
 *
 * Scores take a rotated query: four binary64 lanes (channel i into lane
 * i % 4, products exact), ((l0 + l1) + l2) + l3 rounded to binary32, times
 * the record scale.  Values accumulate in the rotated basis as binary32
 * scale * weight * level, rows in order; one inverse rotation ends a scan.
 *
 * The levels are the reference's published binary32 table; tests/
 * test_oracle_kvq.py pins them to it and to the Gaussian conditional-mean
 * property the table states.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "prism_oracle.h"

#define KVQ_D 256

static uint64_t splitmix(uint64_t *s) {
  *s += 0x9e3779b97f4a7c15ull;
  uint64_t z = *s;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

uint64_t po_kvq_splitmix(uint64_t *state) { return splitmix(state); }

/* The codec's reconstruction levels: the symmetric Gaussian Lloyd-Max
 * levels as the reference publishes them, rounded to binary32 (reference
 * src/kv_quant/tables.rs:10-46; a format table, kept bit for bit).  They lie
 * within 3 ulp of the binary64 fixed point of the conditional-mean iteration,
 * which tests/test_oracle_kvq.py checks; the table, not the iteration, is the
 * codec. */
static const uint32_t kLevels3[8] = {0xc009b97au, 0xbfac0538u, 0xbf418990u, 0xbe7af9f7u,
                                     0x3e7af9f7u, 0x3f418990u, 0x3fac0538u, 0x4009b97au};
static const uint32_t kLevels4[16] = {0xc02ee2bdu, 0xc0046ac7u, 0xbfcf1c25u, 0xbfa0cc2fu,
                                      0xbf713d36u, 0xbf28215bu, 0xbec6ae44u, 0xbe0379fdu,
                                      0x3e0379fdu, 0x3ec6ae44u, 0x3f28215bu, 0x3f713d36u,
                                      0x3fa0cc2fu, 0x3fcf1c25u, 0x40046ac7u, 0x402ee2bdu};

/* `levels` (8 or 16) levels into out[16], the unused slots zero. */
void po_kvq_levels(int levels, float *out) {
  for (int i = 0; i < 16; ++i) {
    uint32_t b = 0;
    if (levels == 8 && i < 8) b = kLevels3[i];
    if (levels == 16) b = kLevels4[i];
    memcpy(&out[i], &b, 4);
  }
}

typedef struct {
  int bits, version;
  uint8_t negative[3][KVQ_D];
  float levels[16];
} kvq_t;

static void kvq_init(kvq_t *q, int bits, uint64_t seed, int version) {
  q->bits = bits;
  q->version = version;
  uint64_t s = seed;
  for (int p = 0; p < 3; ++p)
    for (int i = 0; i < KVQ_D; ++i) q->negative[p][i] = (uint8_t)(splitmix(&s) & 1u);
  po_kvq_levels(bits == 3 ? 8 : 16, q->levels);
}

int po_kvq_record_bytes(int bits) { return bits == 3 ? 100 : bits == 4 ? 132 : 0; }

static int finite_all(const float *x, int n) {
  for (int i = 0; i < n; ++i)
    if (!isfinite(x[i])) return 0;
  return 1;
}

/* The normalised Walsh-Hadamard transform (reference src/kv_quant/
 * scalar.rs:27-47): butterflies of width 1, 2, ..., 128, then 1/16. */
static int hadamard(float *row) {
  float next[KVQ_D];
  memcpy(next, row, sizeof(next));
  for (int half = 1; half < KVQ_D; half *= 2)
    for (int b = 0; b < KVQ_D; b += 2 * half)
      for (int i = b; i < b + half; ++i) {
        const float first = next[i], second = next[i + half];
        next[i] = first + second;
        next[i + half] = first - second;
      }
  for (int i = 0; i < KVQ_D; ++i) next[i] *= 1.0f / 16.0f;
  if (!finite_all(next, KVQ_D)) return PO_E_NONFINITE;
  memcpy(row, next, sizeof(next));
  return PO_OK;
}

static int forward(const kvq_t *q, float *row) {
  for (int p = 0; p < 3; ++p) {
    for (int i = 0; i < KVQ_D; ++i) row[i] *= q->negative[p][i] ? -1.0f : 1.0f;
    const int st = hadamard(row);
    if (st) return st;
  }
  return PO_OK;
}

static int inverse(const kvq_t *q, float *row) {
  for (int p = 2; p >= 0; --p) {
    const int st = hadamard(row);
    if (st) return st;
    for (int i = 0; i < KVQ_D; ++i) row[i] *= q->negative[p][i] ? -1.0f : 1.0f;
  }
  return PO_OK;
}

static int read_code(const uint8_t *codes, int bits, int index) {
  const int offset = index * bits, byte = offset / 8, shift = offset % 8;
  unsigned code = codes[byte] >> shift;
  if (shift + bits > 8) code |= (unsigned)codes[byte + 1] << (8 - shift);
  return (int)(code & ((1u << bits) - 1u));
}

static void write_code(uint8_t *codes, int bits, int index, int code) {
  const int offset = index * bits, byte = offset / 8, shift = offset % 8;
  codes[byte] |= (uint8_t)(code << shift);
  if (shift + bits > 8) codes[byte + 1] |= (uint8_t)(code >> (8 - shift));
}

/* Exhaustive nearest level with the first-code tie rule (reference
 * src/kv_quant/scalar.rs:49-61; the ordered search there gives the same). */
static int nearest(float v, const float *levels, int n) {
  int code = 0;
  float distance = fabsf(v - levels[0]);
  for (int c = 1; c < n; ++c) {
    const float d = fabsf(v - levels[c]);
    if (d < distance) {
      code = c;
      distance = d;
    }
  }
  return code;
}

/* Version 2's guarded scale fit (reference src/kv_quant/fitted_scale.rs). */
static float fitted(const kvq_t *q, const float *row, const uint8_t *codes, float norm_scale) {
  double cross = 0.0, energy = 0.0;
  for (int i = 0; i < KVQ_D; ++i) {
    const double c = (double)q->levels[read_code(codes, q->bits, i)];
    cross = fma((double)row[i], c, cross);
    energy = fma(c, c, energy);
  }
  const float candidate = (float)((double)norm_scale * (cross / energy));
  if (!isfinite(candidate) || candidate <= 0.0f) return norm_scale;
  uint32_t a, b;
  memcpy(&a, &candidate, 4);
  memcpy(&b, &norm_scale, 4);
  if (a == b) return norm_scale;
  double base = 0.0, cand = 0.0;
  for (int i = 0; i < KVQ_D; ++i) {
    const float c = q->levels[read_code(codes, q->bits, i)];
    const float rec = candidate * c;
    if (!isfinite(rec)) return norm_scale;
    const double target = (double)row[i] * (double)norm_scale;
    const double bd = target - (double)(norm_scale * c);
    const double cd = target - (double)rec;
    base = fma(bd, bd, base);
    cand = fma(cd, cd, cand);
  }
  return cand < base ? candidate : norm_scale;
}

/* reference src/kv_quant.rs:515-565 encode */
int po_kvq_encode(int bits, uint64_t seed, int version, const float *input, uint8_t *out) {
  kvq_t q;
  if (!po_kvq_record_bytes(bits)) return PO_E_INVALID;
  kvq_init(&q, bits, seed, version);
  const int len = po_kvq_record_bytes(bits);
  double sq = 0.0;
  for (int i = 0; i < KVQ_D; ++i) {
    if (!isfinite(input[i])) return PO_E_INVALID;
    sq = fma((double)input[i], (double)input[i], sq);
  }
  uint8_t record[132];
  memset(record, 0, sizeof(record));
  if (sq == 0.0) {
    memcpy(out, record, (size_t)len);
    return PO_OK;
  }
  float scale = (float)(sqrt(sq) / 16.0);
  if (!isfinite(scale)) return PO_E_NONFINITE;
  if (scale == 0.0f) return PO_E_INVALID;
  float row[KVQ_D];
  for (int i = 0; i < KVQ_D; ++i) {
    row[i] = (float)((double)input[i] / (double)scale);
    if (!isfinite(row[i])) return PO_E_NONFINITE;
  }
  int st = forward(&q, row);
  if (st) return st;
  uint8_t *codes = record + 4;
  const int n = bits == 3 ? 8 : 16;
  for (int i = 0; i < KVQ_D; ++i) {
    const int code = nearest(row[i], q.levels, n);
    if (!isfinite(scale * q.levels[code])) return PO_E_NONFINITE;
    write_code(codes, bits, i, code);
  }
  if (version == 2) scale = fitted(&q, row, codes, scale);
  memcpy(record, &scale, 4);
  memcpy(out, record, (size_t)len);
  return PO_OK;
}

static int record_scale(int bits, const uint8_t *rec, float *scale) {
  float s;
  memcpy(&s, rec, 4);
  if (!isfinite(s) || signbit(s)) return PO_E_INVALID;
  if (s == 0.0f) {
    for (int i = 4; i < po_kvq_record_bytes(bits); ++i)
      if (rec[i]) return PO_E_INVALID;
  }
  *scale = s;
  return PO_OK;
}

int po_kvq_rotate(int bits, uint64_t seed, const float *input, float *out) {
  kvq_t q;
  kvq_init(&q, bits, seed, 1);
  if (!finite_all(input, KVQ_D)) return PO_E_INVALID;
  float row[KVQ_D];
  memcpy(row, input, sizeof(row));
  const int st = forward(&q, row);
  if (!st) memcpy(out, row, sizeof(row));
  return st;
}

int po_kvq_inverse(int bits, uint64_t seed, float *inout) {
  kvq_t q;
  kvq_init(&q, bits, seed, 1);
  if (!finite_all(inout, KVQ_D)) return PO_E_INVALID;
  float row[KVQ_D];
  memcpy(row, inout, sizeof(row));
  const int st = inverse(&q, row);
  if (!st) memcpy(inout, row, sizeof(row));
  return st;
}

/* reference src/kv_quant/scalar.rs:140-155 dot, times the record scale */
int po_kvq_score(int bits, const float *rotated_query, const uint8_t *rec, float *out) {
  kvq_t q;
  kvq_init(&q, bits, 0, 1);
  float scale;
  int st = record_scale(bits, rec, &scale);
  if (st) return st;
  if (!finite_all(rotated_query, KVQ_D)) return PO_E_INVALID;
  if (scale == 0.0f) {
    *out = 0.0f;
    return PO_OK;
  }
  double lanes[4] = {0.0, 0.0, 0.0, 0.0};
  for (int i = 0; i < KVQ_D; ++i)
    lanes[i % 4] += (double)rotated_query[i] * (double)q.levels[read_code(rec + 4, bits, i)];
  const float unscaled = (float)(((lanes[0] + lanes[1]) + lanes[2]) + lanes[3]);
  if (!isfinite(unscaled)) return PO_E_NONFINITE;
  const float score = unscaled * scale;
  if (!isfinite(score)) return PO_E_NONFINITE;
  *out = score;
  return PO_OK;
}

/* reference src/kv_quant.rs:690-712 accumulate (scalar.rs:157-180) */
int po_kvq_accumulate(int bits, const uint8_t *rec, float weight, float *out) {
  kvq_t q;
  kvq_init(&q, bits, 0, 1);
  if (!finite_all(out, KVQ_D) || !isfinite(weight)) return PO_E_INVALID;
  float scale;
  int st = record_scale(bits, rec, &scale);
  if (st) return st;
  const float ws = weight * scale;
  if (!isfinite(ws)) return PO_E_NONFINITE;
  if (scale == 0.0f) return PO_OK;
  float next[KVQ_D];
  for (int i = 0; i < KVQ_D; ++i) {
    next[i] = out[i] + ws * q.levels[read_code(rec + 4, bits, i)];
    if (!isfinite(next[i])) return PO_E_NONFINITE;
  }
  memcpy(out, next, sizeof(next));
  return PO_OK;
}

int po_kvq_decode(int bits, uint64_t seed, const uint8_t *rec, float *out) {
  float row[KVQ_D];
  memset(row, 0, sizeof(row));
  int st = po_kvq_accumulate(bits, rec, 1.0f, row);
  if (!st) st = po_kvq_inverse(bits, seed, row);
  if (!st) memcpy(out, row, sizeof(row));
  return st;
}

/* One query head over n positions of packed keys and values (reference
 * src/graph/quantized_kv.rs:1294-1338 attend_head, Source arithmetic):
 * query rotated by the key codec, score * attn_scale per position,
 * softmax_round_f16, value scan in position order (a zero weighted scale
 * adds nothing), inverse value rotation, sigmoid gate. */
int po_kvq_attend_head(int kbits, uint64_t kseed, int vbits, uint64_t vseed, const float *query,
                       const uint8_t *keys, const uint8_t *values, size_t n, float attn_scale,
                       const float *gate, float *out) {
  const int kb = po_kvq_record_bytes(kbits), vb = po_kvq_record_bytes(vbits);
  float rq[KVQ_D];
  int st = po_kvq_rotate(kbits, kseed, query, rq);
  if (st) return st;
  float *p = (float *)malloc(sizeof(float) * (n ? n : 1));
  if (!p) return PO_E_INVALID;
  for (size_t t = 0; t < n && !st; ++t) {
    float s;
    st = po_kvq_score(kbits, rq, keys + t * (size_t)kb, &s);
    p[t] = s * attn_scale;
  }
  if (!st) st = po_softmax_round_f16(p, n);
  float acc[KVQ_D];
  memset(acc, 0, sizeof(acc));
  for (size_t t = 0; t < n && !st; ++t) {
    float scale;
    st = record_scale(vbits, values + t * (size_t)vb, &scale);
    if (st) break;
    if (p[t] * scale == 0.0f) continue;
    st = po_kvq_accumulate(vbits, values + t * (size_t)vb, p[t], acc);
  }
  free(p);
  if (!st) st = po_kvq_inverse(vbits, vseed, acc);
  if (st) return st;
  for (int i = 0; i < KVQ_D; ++i) out[i] = acc[i] * po_sigmoid(gate[i]);
  return finite_all(out, KVQ_D) ? PO_OK : PO_E_NONFINITE;
}
