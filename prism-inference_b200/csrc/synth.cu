// synth.cu -- seeded synthetic packed weights (host code).
//
// Benchmark inputs only: the reference has no public weights for this path,
// so random-init weights with the configured distribution stand in for them.
// A counter-based generator (SplitMix64 of seed, stream and byte index) makes
// every tensor reproducible on any host and lets threads fill disjoint row
// ranges independently.
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/prism_b200.h"

namespace {

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

// Round-to-nearest-even binary32 -> binary16 bits (finite inputs).
inline uint16_t to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x477ff000u) return sign | 0x7c00u;
  if (ax >= 0x38800000u) {
    uint32_t h = ((((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13));
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return sign | (uint16_t)h;
  }
  if (ax <= 0x33000000u) return sign;
  uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u, s = 126u - e;
  uint32_t h = m >> s, rem = m & ((1u << s) - 1u), half = 1u << (s - 1u);
  if (rem > half || (rem == half && (h & 1u))) h += 1u;
  return sign | (uint16_t)h;
}

inline float uniform(uint64_t h, float lo, float hi) {
  return lo + (hi - lo) * (float)((h >> 40) * (1.0 / 16777216.0));
}

// 4 codes from one hash: code = floor(16-bit draw * n / 65536)
inline uint8_t pack4(uint64_t h, unsigned n) {
  uint8_t b = 0;
  for (int p = 0; p < 4; ++p) {
    unsigned c = (unsigned)((((h >> (16 * p)) & 0xffffu) * n) >> 16);
    b |= (uint8_t)(c << (2 * p));
  }
  return b;
}

void fill_rows(uint32_t kind, uint64_t r0, uint64_t r1, uint64_t nb, uint64_t seed,
               uint64_t stream, float lo, float hi, uint8_t *out) {
  const int bb = kind == PRISM_B200_KIND_TQ2_0 ? 66 : 84;
  const uint64_t base = splitmix64(seed * 0x2545f4914f6cdd1dull ^ splitmix64(stream + 1));
  for (uint64_t r = r0; r < r1; ++r) {
    for (uint64_t b = 0; b < nb; ++b) {
      uint8_t *blk = out + (r * nb + b) * bb;
      const uint64_t key = base + (r * nb + b) * 128;
      if (kind == PRISM_B200_KIND_TQ2_0) {
        // byte j holds the codes of elements (j/32)*128 + j%32 + 32p, p = 0..3
        for (int j = 0; j < 64; ++j) blk[j] = pack4(splitmix64(key + j), 3);
        uint16_t d = to_half(uniform(splitmix64(key + 64), lo, hi));
        blk[64] = (uint8_t)(d & 0xff);
        blk[65] = (uint8_t)(d >> 8);
      } else {
        for (int j = 0; j < 16; ++j) blk[j] = (uint8_t)(splitmix64(key + 100 + j) >> 56);
        for (int j = 0; j < 64; ++j) blk[16 + j] = pack4(splitmix64(key + j), 4);
        uint16_t d = to_half(uniform(splitmix64(key + 64), lo, hi));
        uint16_t m = to_half(uniform(splitmix64(key + 65), lo * 0.5f, hi * 0.5f));
        blk[80] = (uint8_t)(d & 0xff);
        blk[81] = (uint8_t)(d >> 8);
        blk[82] = (uint8_t)(m & 0xff);
        blk[83] = (uint8_t)(m >> 8);
      }
    }
  }
}

}  // namespace

extern "C" int prism_b200_synth_weights(uint32_t kind, uint64_t rows, uint64_t cols,
                                        uint64_t seed, uint64_t stream, float scale_lo,
                                        float scale_hi, void *out) {
  if ((kind != PRISM_B200_KIND_TQ2_0 && kind != PRISM_B200_KIND_Q2_K) || !out || rows == 0 ||
      cols == 0 || cols % 256 || !(scale_lo > 0.0f) || !(scale_hi >= scale_lo) ||
      scale_hi > 60000.0f)
    return PRISM_B200_E_INVALID;
  const uint64_t nb = cols / 256;
  unsigned threads = std::thread::hardware_concurrency();
  if (threads < 1) threads = 1;
  if (threads > 64) threads = 64;
  if (rows < threads * 16) threads = 1;
  std::vector<std::thread> pool;
  const uint64_t chunk = (rows + threads - 1) / threads;
  for (unsigned t = 0; t < threads; ++t) {
    uint64_t a = t * chunk, b = a + chunk < rows ? a + chunk : rows;
    if (a >= b) break;
    pool.emplace_back(fill_rows, kind, a, b, nb, seed, stream, scale_lo, scale_hi,
                      static_cast<uint8_t *>(out));
  }
  for (auto &th : pool) th.join();
  return PRISM_B200_OK;
}
