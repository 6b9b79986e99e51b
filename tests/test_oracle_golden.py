"""Pin the CPU oracle against the reference's golden vectors.

The fixtures under tests/golden were captured by the reference from the
pinned upstream C ggml kernels (reference tests/tquants.rs:15-77,
tests/kquants.rs:14-72 assert the same fields).  Every comparison here is
bit-exact.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def _bytes(h):
    return np.frombuffer(bytes.fromhex(h), dtype=np.uint8)


@pytest.mark.parametrize("name,kind", [("tq2_0.json", 35), ("q2_k.json", 10),
                                       ("tq1_0.json", 34), ("q3_k.json", 11),
                                       ("q4_k.json", 12), ("q5_k.json", 13),
                                       ("q6_k.json", 14)])
def test_decode_and_generic_dot_match_golden(oracle, name, kind):
    fx = _load(name)
    assert len(fx["cases"]) == 5
    for case in fx["cases"]:
        packed = _bytes(case["OutputHex"])
        decoded = oracle.decode(kind, packed)
        assert decoded.tobytes().hex() == case["DecodedHex"], case["Name"]
        act = np.frombuffer(bytes.fromhex(case["ActivationsHex"]), dtype=oracle.Q8K_DTYPE)
        d = oracle.dot(kind, packed, act)
        assert np.float32(d).tobytes().hex() == case["GenericDotHex"], case["Name"]


def test_tq2_quantizer_matches_golden(oracle):
    for case in _load("tq2_0.json")["cases"]:
        if "InputHex" not in case:
            continue
        x = np.frombuffer(bytes.fromhex(case["InputHex"]), dtype="<f4")
        assert oracle.tq2_quantize(x).tobytes().hex() == case["OutputHex"], case["Name"]


@pytest.mark.parametrize("name,kind", [("tq2_0.json", 35), ("tq1_0.json", 34)])
def test_tq_quantizer_matches_golden(oracle, name, kind):
    n = 0
    for case in _load(name)["cases"]:
        if "InputHex" not in case:
            continue
        x = np.frombuffer(bytes.fromhex(case["InputHex"]), dtype="<f4")
        assert oracle.tq_quantize(kind, x).tobytes().hex() == case["OutputHex"], case["Name"]
        n += 1
    assert n >= 1


def test_q8k_source_and_pinned_rounding_controls(oracle):
    for case in _load("q8k_parity.json")["cases"]:
        x = np.zeros(256, dtype=np.float32)
        x[0] = np.frombuffer(bytes.fromhex(case["input_bits"][0]), dtype=">f4")[0]
        x[1] = np.frombuffer(bytes.fromhex(case["input_bits"][1]), dtype=">f4")[0]
        src = oracle.q8k_quantize(x, pinned=False)
        assert int(src["values"][0][1]) == case["source_code_at_1"]
        pinned = oracle.q8k_quantize(x, pinned=True)
        assert int(pinned["values"][0][1]) == case["native_code_at_1"]
        assert pinned.tobytes().hex() == case["native_block_hex"]
        iscale = np.float32(-127.0) / x[0]
        assert np.float32(iscale).tobytes()[::-1].hex() == case["inverse_scale_bits"]


def test_half_conversions_exhaustive(oracle):
    L = oracle.lib()
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    ours = np.array([L.po_half_to_float(int(b)) for b in bits], dtype=np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(ours[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.all(np.isnan(ours[np.isnan(ref)]))
    # float -> half: numpy's conversion is IEEE round-to-nearest-even
    rng = np.random.default_rng(0)
    xs = np.concatenate([
        rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32).view(np.float32),
        (np.arange(-70000, 70000, 0.25, dtype=np.float32)),
        np.array([65504, 65519.996, 65520, 2**-24, 2**-25, 2**-25 * 1.0001, 3 * 2**-26, 6.1e-5], dtype=np.float32),
    ])
    xs = xs[~np.isnan(xs)]
    ref16 = xs.astype(np.float16).view(np.uint16)
    ours16 = np.array([L.po_float_to_half(float(v)) for v in xs[:50000]], dtype=np.uint16)
    assert np.array_equal(ours16, ref16[:50000])
    # NaN becomes the canonical quiet NaN with its sign
    assert L.po_float_to_half(float("nan")) & 0x7fff == 0x7e00


def test_q8k_properties(oracle):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4096).astype(np.float32)
    blocks = oracle.q8k_quantize(x)
    for b, blk in enumerate(blocks):
        c = x[b * 256:(b + 1) * 256]
        m = c[np.argmax(np.abs(c))]
        iscale = np.float32(-127.0) / m
        assert blk["scale"] == np.float32(1.0) / iscale
        q = np.minimum(np.rint(c * iscale), 127).astype(np.int8)
        assert np.array_equal(blk["values"], q)
        assert np.array_equal(blk["sums"], q.reshape(16, 16).astype(np.int32).sum(1))
    # an all-zero block is the zero block
    z = oracle.q8k_quantize(np.zeros(256, np.float32))
    assert z["scale"][0] == 0 and not z["values"].any()


def test_block_dots_recompose_dot(oracle):
    """The f32 dot is the sequential chain over the exact block integers."""
    rng = np.random.default_rng(5)
    nb = 16
    w = np.zeros(nb * 66, np.uint8)
    for b in range(nb):
        w[b * 66:b * 66 + 64] = rng.integers(0, 256, 64)
        w[b * 66 + 64:b * 66 + 66] = np.frombuffer(np.float16(rng.uniform(0.01, 0.05)).tobytes(), np.uint8)
    act = oracle.q8k_quantize(rng.standard_normal(nb * 256).astype(np.float32))
    ints = oracle.block_dots(35, w, act)
    s = np.float32(0)
    for b in range(nb):
        d = np.frombuffer(w[b * 66 + 64:b * 66 + 66].tobytes(), np.float16)[0].astype(np.float32)
        s = np.float32(s + np.float32(np.float32(ints[b]) * np.float32(d * act["scale"][b])))
    assert s == oracle.dot(35, w, act)
    dec = oracle.decode(35, w)
    vals = act["values"].reshape(-1).astype(np.int64)
    codes = np.rint(dec.reshape(nb, 256) / np.array(
        [np.frombuffer(w[b * 66 + 64:b * 66 + 66].tobytes(), np.float16)[0] for b in range(nb)],
        dtype=np.float32)[:, None]).astype(np.int64)
    assert np.array_equal(ints, (codes * vals.reshape(nb, 256)).sum(1))


def test_matvec_threads_bit_equal(oracle):
    rng = np.random.default_rng(7)
    rows, cols = 37, 512
    for kind in (35, 10):
        bb = oracle.block_bytes(kind)
        w = rng.integers(0, 256, rows * cols // 256 * bb).astype(np.uint8).reshape(rows, -1, bb)
        if kind == 35:
            w[:, :, 64:66] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
        else:
            w[:, :, 80:82] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
            w[:, :, 82:84] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
        act = oracle.q8k_quantize(rng.standard_normal(cols).astype(np.float32))
        y1 = oracle.matvec(kind, w, rows, cols, act, threads=1)
        y5 = oracle.matvec(kind, w, rows, cols, act, threads=5)
        assert np.array_equal(y1.view(np.uint32), y5.view(np.uint32))
        for r in (0, 17, 36):
            assert y1[r] == oracle.dot(kind, w[r].reshape(-1), act)


def test_project_tokens_equals_per_token_matvec(oracle):
    rng = np.random.default_rng(8)
    rows, cols, tokens = 45, 768, 70   # more than two 32-token tiles
    for kind in (35, 10):
        bb = oracle.block_bytes(kind)
        w = rng.integers(0, 256, rows * cols // 256 * bb).astype(np.uint8).reshape(rows, -1, bb)
        if kind == 35:
            w[:, :, 64:66] = np.frombuffer(np.float16(0.03).tobytes(), np.uint8)
        else:
            w[:, :, 80:82] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
            w[:, :, 82:84] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
        x = rng.standard_normal((tokens, cols)).astype(np.float32)
        for pinned in (False, True):
            y = oracle.project_tokens(kind, w, rows, cols, x, pinned, threads=4)
            for t in (0, 31, 32, 69):
                ref = oracle.matvec(kind, w, rows, cols, oracle.q8k_quantize(x[t], pinned))
                assert np.array_equal(y[t].view(np.uint32), ref.view(np.uint32))
