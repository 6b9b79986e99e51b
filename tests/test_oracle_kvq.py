"""The oracle's rotated scalar KV codec (the reference's "rsq" profile,
src/kv_quant.rs and src/kv_quant/), pinned.

  * the binary32 level tables bit for bit against the reference's published
    tables (tests/golden/kvq_reference.json, extracted from
    src/kv_quant/tables.rs), and the Gaussian conditional-mean property they
    state (src/kv_quant/tests.rs codebook_centroids_satisfy_...);
  * the SplitMix64 words of seed 0 and the little-endian 3- and 4-bit
    packing goldens (src/kv_quant/tests.rs:396-420);
  * the transform against an independent dense signed Hadamard product, and
    its inverse (src/kv_quant/tests.rs:424-456);
  * score and accumulation against an independent reconstruction, bit for
    bit (src/kv_quant/tests.rs:488-537);
  * encode's norm scale and fixture error bounds, version 2's fitted scale,
    the canonical zero record and malformed-record refusals
    (src/kv_quant/tests.rs:539-745);
  * packed attention against dense attention over the decoded rows.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
KEY = 0x5357_4946_544b_5631
VALUE = 0x5357_4946_5456_5631


@pytest.fixture(scope="module")
def ref():
    with open(os.path.join(HERE, "golden", "kvq_reference.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def o():
    from oracle import oracle
    return oracle


def input_row():
    """The reference's codec fixture row: (i - 127.5)/32 + sin(0.17 (i - 127.5))
    in binary32 arithmetic."""
    linear = np.arange(256, dtype=np.float32) - np.float32(127.5)
    return (linear / np.float32(32.0) + np.sin(linear * np.float32(0.17))).astype(np.float32)


def splitmix(state):
    mask = (1 << 64) - 1
    state = (state + 0x9E3779B97F4A7C15) & mask
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
    return state, z ^ (z >> 31)


def sign_passes(seed):
    s, out = seed, np.zeros((3, 256), bool)
    for p in range(3):
        for i in range(256):
            s, w = splitmix(s)
            out[p, i] = bool(w & 1)
    return out


def record(bits, scale, levels):
    """A record whose code i is i % levels, built one bit at a time."""
    n = 4 + 256 * bits // 8
    rec = np.zeros(n, np.uint8)
    rec[:4] = np.frombuffer(np.float32(scale).tobytes(), np.uint8)
    for i in range(256):
        code = i % levels
        for b in range(bits):
            sb = i * bits + b
            if code & (1 << b):
                rec[4 + sb // 8] |= 1 << (sb % 8)
    return rec


def test_levels_match_the_published_tables(o, ref):
    assert o.kvq_levels(3).view(np.uint32).tolist() == ref["three_bits"]
    assert o.kvq_levels(4).view(np.uint32).tolist() == ref["four_bits"]


def test_levels_are_gaussian_conditional_means(o):
    for bits, n in ((3, 8), (4, 16)):
        t = o.kvq_levels(bits)[:n].astype(np.float64)
        assert np.all(np.diff(t) > 0) and np.array_equal(t, -t[::-1])
        for i in range(n):
            left = -10.0 if i == 0 else 0.5 * (t[i - 1] + t[i])
            right = 10.0 if i == n - 1 else 0.5 * (t[i] + t[i + 1])
            x = left + (np.arange(4096) + 0.5) * (right - left) / 4096
            d = np.exp(-0.5 * x * x)
            assert abs(np.sum(x * d) / np.sum(d) - t[i]) < 2e-6


def test_splitmix_known_words(o, ref):
    import ctypes
    s = ctypes.c_uint64(0)
    got = [o.lib().po_kvq_splitmix(ctypes.byref(s)) for _ in range(3)]
    assert got == ref["splitmix_seed0"]
    st, words = 0, []
    for _ in range(3):
        st, w = splitmix(st)
        words.append(w)
    assert words == ref["splitmix_seed0"]


def test_packing_goldens_and_code_reads(o, ref):
    for bits, levels, golden in ((3, 8, ref["pack3"]), (4, 16, ref["pack4"])):
        rec = record(bits, 1.0, levels)
        assert rec[4:4 + len(golden)].tolist() == golden
        out = np.zeros(256, np.float32)
        o.kvq_accumulate(bits, rec, 1.0, out)
        assert np.array_equal(out, o.kvq_levels(bits)[np.arange(256) % levels])
    assert o.kvq_record_bytes(3) == 100 and o.kvq_record_bytes(4) == 132


def dense_rotation(x, seed):
    h = np.array([[(-1.0) ** bin(i & j).count("1") for j in range(256)] for i in range(256)])
    row = x.astype(np.float64)
    for signs in sign_passes(seed):
        row = (h @ (row * np.where(signs, -1.0, 1.0)) / 16.0).astype(np.float32).astype(np.float64)
    return row


def test_transform_matches_a_dense_signed_hadamard(o):
    x = input_row()
    got = o.kvq_rotate(4, 42, x)
    assert np.max(np.abs(got - dense_rotation(x, 42))) < 4e-6
    assert np.max(np.abs(o.kvq_inverse(4, 42, got) - x)) < 4e-6


def test_score_and_accumulate_match_independent_reconstruction(o):
    q = input_row()
    for bits, levels in ((3, 8), (4, 16)):
        t = o.kvq_levels(bits)
        rec = record(bits, 2.0, levels)
        c = t[np.arange(256) % levels]
        lanes = [0.0] * 4
        for i in range(256):
            lanes[i % 4] += float(q[i]) * float(c[i])
        want = np.float32(((lanes[0] + lanes[1]) + lanes[2]) + lanes[3]) * np.float32(2.0)
        assert o.kvq_score(bits, q, rec).view(np.uint32) == want.view(np.uint32)
        acc = np.zeros(256, np.float32)
        o.kvq_accumulate(bits, rec, 1.0, acc)
        assert np.array_equal(acc, c * np.float32(2.0))
        dec = o.kvq_decode(bits, 91, rec)[0]
        assert np.max(np.abs(o.kvq_rotate(bits, 91, dec) - c * 2)) < 4e-6
    # weighted rows accumulate in the rotated basis, rows in order
    t = o.kvq_levels(4)[np.arange(256) % 16]
    acc = np.zeros(256, np.float32)
    o.kvq_accumulate(4, record(4, 2.0, 16), 0.25, acc)
    o.kvq_accumulate(4, record(4, 0.5, 16), 0.75, acc)
    assert np.array_equal(acc, np.float32(0.5) * t + np.float32(0.375) * t)


def test_encode_keeps_the_norm_scale_and_bounds_the_error(o):
    x = input_row()
    norm2 = float(np.sum(x.astype(np.float64) ** 2))
    for bits, bound in ((3, 0.12), (4, 0.04)):
        rec = o.kvq_encode(bits, 42, x)[0]
        scale = rec[:4].view(np.float32)[0]
        assert abs(scale - np.float32(np.sqrt(norm2) / 16)) <= 1e-6 * scale
        dec = o.kvq_decode(bits, 42, rec)[0]
        assert np.sum((x.astype(np.float64) - dec) ** 2) / norm2 < bound


def rotated_error(o, bits, x, baseline, rec):
    s = baseline[:4].view(np.float32)[0]
    normalized = (x.astype(np.float64) / np.float64(s)).astype(np.float32)
    target = o.kvq_rotate(bits, 42, normalized)
    recon = np.zeros(256, np.float32)
    o.kvq_accumulate(bits, rec, 1.0, recon)
    return float(np.sum((target.astype(np.float64) * np.float64(s) - recon) ** 2))


def test_fitted_scale_keeps_codes_and_never_raises_the_error(o):
    sparse = np.zeros(256, np.float32)
    sparse[19] = 3.0
    fixtures = [input_row(), sparse, np.ones(256, np.float32),
                (input_row() * np.float32(1e-39)).astype(np.float32),
                (input_row() * np.float32(1e30)).astype(np.float32)]
    improved = 0
    for bits in (3, 4):
        for x in fixtures:
            base = o.kvq_encode(bits, 42, x, version=1)[0]
            fit = o.kvq_encode(bits, 42, x, version=2)[0]
            assert np.array_equal(fit[4:], base[4:])
            before = rotated_error(o, bits, x, base, base)
            after = rotated_error(o, bits, x, base, fit)
            assert after <= before * (1 + 1e-12)
            improved += after < before
    assert improved > 0


def test_canonical_zero_and_malformed_records(o):
    from oracle.oracle import OracleError
    for bits in (3, 4):
        z = o.kvq_encode(bits, 42, np.zeros(256, np.float32))[0]
        assert not z.any()
        q = input_row()
        assert o.kvq_score(bits, q, z) == 0.0
        bad = z.copy()
        bad[4] = 1
        with pytest.raises(OracleError):
            o.kvq_score(bits, q, bad)
        for s in (-0.0, np.nan, np.inf, -1.0):
            r = record(bits, 1.0, 8)
            r[:4] = np.frombuffer(np.float32(s).tobytes(), np.uint8)
            with pytest.raises(OracleError):
                o.kvq_score(bits, q, r)
        with pytest.raises(OracleError):
            x = input_row().copy()
            x[7] = np.nan
            o.kvq_encode(bits, 42, x)
        with pytest.raises(OracleError):   # a nonzero row whose scale underflows
            x = np.zeros(256, np.float32)
            x[0] = np.float32(1e-45)
            o.kvq_encode(bits, 42, x)


@pytest.mark.parametrize("policy", ["rsq4", "rsq4vf", "rsq4k3v"])
def test_packed_attention_tracks_dense_attention_over_decoded_rows(o, policy):
    kb, vb, ver = o.KVQ_POLICIES[policy]
    rng = np.random.default_rng(5)
    n, heads, kvh = 37, 4, 2
    k = rng.standard_normal((n, kvh, 256)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((n, kvh, 256)).astype(np.float16).astype(np.float32)
    q = rng.standard_normal((heads, 256)).astype(np.float16).astype(np.float32)
    g = rng.standard_normal((heads, 256)).astype(np.float32)
    keys = o.kvq_encode(kb, KEY, k.reshape(-1, 256)).reshape(n, kvh, -1)
    vals = o.kvq_encode(vb, VALUE, v.reshape(-1, 256), version=ver).reshape(n, kvh, -1)
    got = o.kvq_attend(policy, q, keys, vals, heads, kvh, 1 / 16, g)
    kd = o.kvq_decode(kb, KEY, keys.reshape(-1, kb * 32 + 4)).reshape(n, kvh, 256)
    vd = o.kvq_decode(vb, VALUE, vals.reshape(-1, vb * 32 + 4)).reshape(n, kvh, 256)
    for h in range(heads):
        s = kd[:, h // 2] @ q[h].astype(np.float64) / 16
        p = np.exp(s - s.max())
        p /= p.sum()
        want = (p @ vd[:, h // 2]) / (1 + np.exp(-g[h].astype(np.float64)))
        # binary16 probabilities and binary32 rotation rounding
        assert np.max(np.abs(got[h] - want)) < 2e-3 * max(1.0, np.max(np.abs(want)))
