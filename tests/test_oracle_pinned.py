"""The oracle's GDN, attention and RoPE arithmetic pinned to the reference's
native captures.

The reference pins its pinned ("Swift") arithmetic with native ggml
captures and shows that its Source arithmetic -- the contract every
synthetic model, and so every kernel of this library, follows -- differs
from them only in summation order and fusing (reference src/graph.rs:
6481-6556, 7976-8024; src/kernels/pinned_attention.rs:1394-1578).  The
oracle restates both variants; this test checks the pinned restatement bit
for bit against every capture (tests/golden/pinned.json, extracted by
tests/golden/make_golden.py) and repeats the reference's own contrasts:

  * GDN: the pinned dot and row update reproduce the native dot, output and
    updated state row; the Source row (binary64 dot sums, separately rounded
    update) does not, on these cancellation-heavy rows -- as the reference
    asserts -- but stays within the binary32 rounding of the terms;
  * attention dots and the masked softmax (through the restated native
    vector exponential) reproduce the native bits; Source dots and softmax
    agree to the terms' rounding;
  * RoPE, out of place and in place, reproduces the native rotation from
    the native cos/sin; Source RoPE differs, as the reference asserts.

The captures share the Source path's structure (which operands meet in
which order of the row update, which pairs rotate, which values the
softmax normalises), so pinning them pins the oracle's Source GDN,
attention and RoPE up to that stated reduction order.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def cap():
    with open(os.path.join(HERE, "golden", "pinned.json")) as f:
        return json.load(f)


def f32(bits):
    return np.array(bits, np.uint32).view(np.float32)


def b32(x):
    return np.asarray(x, np.float32).reshape(-1).view(np.uint32).tolist()


def half_to_f32(bits):
    return np.array(bits, np.uint16).view(np.float16).astype(np.float32)


def source_dot(a, b):
    """The reference's Source float_dot: binary32 products summed in binary64."""
    from oracle import oracle
    return np.float32(oracle.float_dot(np.asarray(a, np.float32), np.asarray(b, np.float32)))


def term_bound(a, b):
    """Bound of a reordering: n * eps(binary32) * sum |a_i b_i|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return len(a) * 2.0 ** -23 * float(np.sum(np.abs(a * b)))


def test_gdn_dot_and_rows(cap):
    from oracle import oracle
    for d in cap["gdn"]["dots"]:
        x, y = f32(d["x"]), f32(d["y"])
        assert b32(oracle.pinned_gdn_dot(x, y)) == [d["native"]]
        src = source_dot(x, y)
        assert b32(src) != [d["native"]]  # the reference's assert_ne (cancellation-heavy)
        assert abs(float(src) - float(f32([d["native"]])[0])) <= term_bound(x, y)
    scale = np.float32(1.0) / np.sqrt(np.float32(128.0))
    for r in cap["gdn"]["rows"]:
        v = f32([r["v"]])[0]
        q, k, st = f32(r["q"]), f32(r["k"]), f32(r["state"])
        # pinned: delta = v - dot(S, k); S += delta * k (fused); out = dot(S, q) / sqrt(d)
        delta = np.float32(v - oracle.pinned_gdn_dot(st, k))
        new = oracle.pinned_gdn_add_scaled(st, k, delta)
        out = np.float32(oracle.pinned_gdn_dot(new, q) * scale)
        assert b32(new) == r["native_state"]
        assert b32(out) == [r["native_out"]]
        # Source: binary64 dot sums, separately rounded update
        sdelta = np.float32(v - source_dot(st, k))
        snew = (st + np.float32(sdelta) * k).astype(np.float32)
        sout = np.float32(source_dot(snew, q) * scale)
        assert b32(sout) != [r["native_out"]]  # the reference's assert_ne
        assert abs(float(sout) - float(out)) <= term_bound(new, q) * float(scale) * 4


def test_attention_dots_and_weighted_value(cap):
    from oracle import oracle
    for c in cap["attention_dot"]["cases"]:
        a, b = f32(c["first"]), f32(c["second"])
        assert b32(oracle.pinned_attention_dot(a, b)) == [c["native"]], c["name"]
        src = source_dot(a, b)
        assert abs(float(src) - float(f32([c["native"]])[0])) <= term_bound(a, b), c["name"]
    w = cap["attention_dot"]["weighted_value"]
    vals = half_to_f32(w["value_half_bits"])
    probs = half_to_f32(w["probability_half_bits"])
    assert b32(oracle.pinned_attention_dot(vals, probs)) == [w["native_bits"]]


def test_masked_softmax(cap):
    from oracle import oracle
    for c in cap["softmax"]:
        x = f32(c["input"])
        got = oracle.pinned_softmax(x)
        assert b32(got) == c["native"], len(x)
        # rounding to binary16 fused into the scaling pass equals rounding after it
        fused = oracle.pinned_softmax(x, round_f16=True)
        assert b32(fused) == b32(got.astype(np.float16).astype(np.float32))
        # Source softmax (libm exponential, binary64 total): the same
        # probabilities to the exponential's rounding
        src = np.exp((x - x.max()).astype(np.float64)).astype(np.float32)
        src = (src * np.float32(1.0 / np.sum(src.astype(np.float64)))).astype(np.float32)
        assert np.max(np.abs(src - got)) <= 4e-7


def test_vector_exp_tracks_the_exponential():
    from oracle import oracle
    for x in np.linspace(-80.0, 0.0, 2001, dtype=np.float32):
        got = float(oracle.vector_exp(x))
        want = float(np.exp(np.float64(x)))
        # the degree-5 polynomial's own error stays under 2 ulp over the range
        assert abs(got - want) <= 2 * float(np.spacing(np.float32(want))), x
    for x in (-100.0, -150.0, -200.0):  # the underflow branches stay tiny and non-negative
        assert 0.0 <= float(oracle.vector_exp(x)) < 1e-38


def test_rope_out_of_place_and_in_place(cap):
    from oracle import oracle
    r = cap["rope"]
    x = f32(r["input"])
    for c in r["cases"]:
        cs = np.empty(2 * len(c["cos"]), np.float32)
        cs[0::2], cs[1::2] = f32(c["cos"]), f32(c["sin"])
        out = oracle.pinned_rope(x, cs, head=r["head"], rotary=r["rotary"])
        assert b32(out) == c["native_out_of_place"], c["position"]
        inplace = oracle.pinned_rope(x, cs, head=r["head"], rotary=r["rotary"], in_place=True)
        assert b32(inplace[:64]) == c["native_in_place_first64"], c["position"]
        assert b32(inplace[64:]) == b32(x[64:])
        src = oracle.source_rope(x, cs, head=r["head"], rotary=r["rotary"])
        assert b32(src) != c["native_out_of_place"]  # the reference's assert_ne
        assert np.max(np.abs(src - out)) <= 4 * 2.0 ** -23 * np.max(np.abs(x)) * 2
    bd = r["boundary"]
    cs = np.tile(np.array([1.0, 0.0], np.float32), 32)
    cs[2 * bd["pair"]], cs[2 * bd["pair"] + 1] = f32([bd["cos"]])[0], f32([bd["sin"]])[0]
    v = np.zeros(256, np.float32)
    v[bd["pair"]], v[bd["pair"] + 32] = f32([bd["first"]])[0], f32([bd["second"]])[0]
    ip = oracle.pinned_rope(v, cs, in_place=True)
    op = oracle.pinned_rope(v, cs)
    assert b32(ip[[bd["pair"], bd["pair"] + 32]]) == [bd["in_place_0"], bd["in_place_1"]]
    assert b32(op[[bd["pair"], bd["pair"] + 32]]) == [bd["out_of_place_0"], bd["out_of_place_1"]]
    halves = ip[[bd["pair"], bd["pair"] + 32]].astype(np.float16).view(np.uint16).astype(np.uint32)
    assert int(halves[0] | (halves[1] << 16)) == bd["half_words"]


def capture_head(r, rows=128, seed=0):
    """A one-token head holding a native capture row as state row 0 (the
    other rows random), with decay = beta = 1: the pinned step of that row
    is then exactly the capture's recipe."""
    rng = np.random.default_rng(seed)
    d = len(r["q"])
    state = (rng.standard_normal((1, 1, rows, d)) * 0.05).astype(np.float32)
    state[0, 0, 0] = f32(r["state"])
    q = f32(r["q"]).reshape(1, 1, 1, d)
    k = f32(r["k"]).reshape(1, 1, 1, d)
    v = rng.standard_normal((1, 1, 1, rows)).astype(np.float32)
    v[0, 0, 0, 0] = f32([r["v"]])[0]
    one = np.ones((1, 1, 1), np.float32)
    return state, q, k, v, one, one


def test_pinned_head_step_reproduces_the_native_rows(cap):
    """The pinned GDN recurrence over a head (the reference's
    step_row_in_place per row and token, src/kernels/pinned_gdn.rs:370-455)
    gives the native capture's updated state row and output bit for bit."""
    from oracle import oracle
    for i, r in enumerate(cap["gdn"]["rows"]):
        state, q, k, v, g, b = capture_head(r, seed=i)
        rc, new, out = oracle.pinned_gdn_prefill(state, q, k, v, g, b)
        assert rc == 0
        assert b32(new[0, 0, 0]) == r["native_state"]
        assert b32(out[0, 0, 0, 0]) == [r["native_out"]]


def test_pinned_head_step_tokens_and_rows():
    """Over several tokens the pinned recurrence of a row equals the row
    stepped alone token by token, with the decay and beta applied as the
    reference's step_row_in_place does (unfused multiplies around the
    pinned dots); heads share key heads by h % key_heads."""
    from oracle import oracle
    rng = np.random.default_rng(3)
    B, T, H, KH, d = 2, 5, 4, 2, 128
    q = rng.standard_normal((B, T, KH, d)).astype(np.float32)
    k = rng.standard_normal((B, T, KH, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, H, d)).astype(np.float32)
    g = rng.uniform(0.5, 1.0, (B, T, H)).astype(np.float32)
    bt = rng.uniform(0.1, 0.9, (B, T, H)).astype(np.float32)
    s0 = (rng.standard_normal((B, H, d, d)) * 0.1).astype(np.float32)
    rc, s, o = oracle.pinned_gdn_prefill(s0, q, k, v, g, bt)
    assert rc == 0
    scale = np.float32(1.0) / np.sqrt(np.float32(d))
    for b, h, r in [(0, 0, 0), (1, 3, 77), (1, 2, 127)]:
        row = s0[b, h, r].copy()
        for t in range(T):
            kk, qq = k[b, t, h % KH], q[b, t, h % KH]
            row = (row * g[b, t, h]).astype(np.float32)
            dk = oracle.pinned_gdn_dot(row, kk)
            delta = np.float32(np.float32(v[b, t, h, r] - dk) * bt[b, t, h])
            row = oracle.pinned_gdn_add_scaled(row, kk, delta)
            assert b32(o[b, t, h, r]) == b32(np.float32(oracle.pinned_gdn_dot(row, qq) * scale))
        assert b32(s[b, h, r]) == b32(row)
