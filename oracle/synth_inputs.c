/*
 * synth_inputs.c -- seeded synthetic packed weights for the CPU side.
 *
 * TEST INFRASTRUCTURE ONLY.  The benchmark's reference arm builds its
 * random-init model here, so that timing the CPU restatement never maps the
 * product library.  The generator is a counter-based SplitMix64 of (seed,
 * stream, byte index); it yields the same bytes as the product library's
 * seeded generator (prism_b200_synth_weights), which tests/test_abi_cpu.py
 * checks byte for byte.  The value distributions are the benchmark
 * configurations' (codes uniform in {0,1,2} for TQ2_0, i.e. weights in
 * {-1,0,+1}; 2-bit quants uniform in 0..3 and random 4-bit scale/min
 * nibbles for Q2_K; binary16 block scales uniform in [lo, hi)).
 */
#include <string.h>

#include "prism_oracle.h"

static inline uint64_t sm64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

/* A value uniform in [lo, hi) from the top 24 bits of a hash. */
static inline float draw_uniform(uint64_t h, float lo, float hi) {
  return lo + (hi - lo) * (float)((double)(h >> 40) * (1.0 / 16777216.0));
}

/* Four 2-bit codes, each floor(16-bit draw * n / 65536), packed low first. */
static inline uint8_t four_codes(uint64_t h, unsigned n) {
  uint8_t b = 0;
  for (int p = 0; p < 4; ++p) {
    const unsigned c = (unsigned)((((h >> (16 * p)) & 0xffffu) * n) >> 16);
    b |= (uint8_t)(c << (2 * p));
  }
  return b;
}

int po_synth_weights(uint32_t kind, uint64_t rows, uint64_t cols, uint64_t seed,
                     uint64_t stream, float lo, float hi, uint8_t *out) {
  if ((kind != 35 && kind != 10) || !out || rows == 0 || cols == 0 || cols % 256 ||
      !(lo > 0.0f) || !(hi >= lo) || hi > 60000.0f)
    return PO_E_INVALID;
  const uint64_t nb = cols / 256;
  const int bb = kind == 35 ? 66 : 84;
  const uint64_t base = sm64(seed * 0x2545f4914f6cdd1dull ^ sm64(stream + 1));
  for (uint64_t u = 0; u < rows * nb; ++u) {
    uint8_t *blk = out + u * bb;
    const uint64_t key = base + u * 128;
    if (kind == 35) {
      /* byte j holds the codes of elements (j/32)*128 + j%32 + 32p, p = 0..3 */
      for (int j = 0; j < 64; ++j) blk[j] = four_codes(sm64(key + j), 3);
      const uint16_t d = po_float_to_half(draw_uniform(sm64(key + 64), lo, hi));
      blk[64] = (uint8_t)(d & 0xff);
      blk[65] = (uint8_t)(d >> 8);
    } else {
      for (int j = 0; j < 16; ++j) blk[j] = (uint8_t)(sm64(key + 100 + j) >> 56);
      for (int j = 0; j < 64; ++j) blk[16 + j] = four_codes(sm64(key + j), 4);
      const uint16_t d = po_float_to_half(draw_uniform(sm64(key + 64), lo, hi));
      const uint16_t m = po_float_to_half(draw_uniform(sm64(key + 65), lo * 0.5f, hi * 0.5f));
      blk[80] = (uint8_t)(d & 0xff);
      blk[81] = (uint8_t)(d >> 8);
      blk[82] = (uint8_t)(m & 0xff);
      blk[83] = (uint8_t)(m >> 8);
    }
  }
  return PO_OK;
}
