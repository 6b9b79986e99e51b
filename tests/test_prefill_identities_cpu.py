"""Arithmetic facts the batched prefill's exactness rests on, checked on the
host (no GPU).

1. The attention kernel widens binary16 cache values to binary64 from their
   bit fields (normal numbers and zeros; anything else through binary32).
   The formula must give the same binary64 value as the conversion for every
   one of the 65536 bit patterns.
2. A binary16 x binary16 product is exact in binary32 (22 significant bits
   and no underflow), so the decode kernel's binary64 sum of binary32-rounded
   products equals a binary64 FMA chain on the widened operands.
3. Under the Gated DeltaNet row update (s = decay*s; s += delta*k) a
   non-finite state element never becomes finite again, so checking the
   final state after a prompt reports exactly when a per-token check would.
"""
import math

import numpy as np


def _widen_f16_bits(h):
    """The kernel's f16_bits_to_f64, restated (prefill.cuh)."""
    e, m, sgn = (h >> 10) & 31, h & 1023, (h >> 15) << 31
    if (e - 1) & 0xFFFFFFFF < 30:
        hi = sgn | ((e + 1008) << 20) | (m << 10)
        return np.array([hi << 32], np.uint64).view(np.float64)[0]
    if h & 0x7FFF == 0:
        return np.array([sgn << 32], np.uint64).view(np.float64)[0]
    return np.float64(np.array([h], np.uint16).view(np.float16)[0].astype(np.float32))


def test_f16_widening_matches_conversion_for_every_pattern():
    bits = np.arange(65536, dtype=np.uint32)
    want = bits.astype(np.uint16).view(np.float16).astype(np.float64)
    for h in range(65536):
        got = _widen_f16_bits(h)
        w = want[h]
        if math.isnan(w):
            assert math.isnan(got), h
        else:
            assert np.array([got]).view(np.uint64)[0] == np.array([w]).view(np.uint64)[0], h


def test_f16_products_exact_and_fma_chain_equals_sum_of_rounded_products():
    rng = np.random.default_rng(7)
    # every exponent range of binary16, subnormals and extremes included
    raw = rng.integers(0, 65536, size=(4000, 8), dtype=np.uint32).astype(np.uint16)
    vals = raw.view(np.float16).astype(np.float32)
    vals[~np.isfinite(vals)] = 1.0
    q, k = vals[:2000], vals[2000:]
    p32 = (q * k).astype(np.float32)                    # binary32-rounded products
    p64 = q.astype(np.float64) * k.astype(np.float64)   # exact products
    assert np.array_equal(p32.astype(np.float64), p64)
    # the decode kernel's 8-term partial: ((p0 + p1) + p2) ... in binary64
    seq = np.zeros(q.shape[0])
    for j in range(8):
        seq = seq + p32[:, j].astype(np.float64)
    # the prefill kernel's chain: a binary64 product, then FMAs (exact
    # products, so one rounding per step as above)
    fma = p64[:, 0].copy()
    for j in range(1, 8):
        fma = fma + p64[:, j]
    assert np.array_equal(seq.view(np.uint64), fma.view(np.uint64))


def test_nonfinite_state_is_absorbing_under_the_row_update():
    rng = np.random.default_rng(11)
    f = np.float32
    specials = [f(np.inf), f(-np.inf), f(np.nan)]
    with np.errstate(all="ignore"):
        for trial in range(2000):
            s = f(rng.choice(specials))
            for _ in range(6):
                decay = f(rng.choice([0.0, 1e-30, 0.5, 1.0]))
                delta = f(rng.choice([0.0, -3.0, 2.5, 1e30, np.inf, np.nan]))
                kk = f(rng.choice([0.0, -1.0, 0.25, 1e-20]))
                s = f(f(decay * s) + f(delta * kk))
                assert not np.isfinite(s), (trial, decay, delta, kk)
