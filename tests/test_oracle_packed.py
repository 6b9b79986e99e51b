"""The oracle's PQ2 (type 142) and PTQ1 (type 143) restatement, pinned.

  * the native C++ codec capture (tests/golden/ptq_reference.json, from the
    reference's tests/fixtures/ptq-reference.bin): for all 161 cases, every
    PTQ block decodes to the same 128 weights as its PQ2 twin and carries the
    same scale, and the binary16 conversions match the captured bits;
  * the reference's own known answers for the two activation contracts
    (reference tests/kernels.rs:206-320): Q8_K ties to even with per-half
    scales for PQ2, Q8_0 rounding away from zero with 32-wide binary16
    scales for PTQ1 and for PQ2 rows that are not a multiple of 256 wide,
    the native code 3 (+2), zero scales and zero activations.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def cap():
    with open(os.path.join(HERE, "golden", "ptq_reference.json")) as f:
        return json.load(f)


def pq2(scale, symbols):
    """A PQ2 block: every weight 0 (code 1) except the given (index, code)
    (the reference's test helper, tests/kernels.rs:27-36)."""
    b = bytearray([0x55] * 34)
    b[0:2] = int(scale).to_bytes(2, "little")
    for index, symbol in symbols:
        shift = 2 * (index % 4)
        b[2 + index // 4] &= ~(3 << shift) & 0xFF
        b[2 + index // 4] |= symbol << shift
    return bytes(b)


def pack_ptq(block):
    """PQ2 -> PTQ1 (reference tools/ternary/src/lib.rs:159-188): five codes
    per byte in base 3 for weights 0-119 (two widths, 16 and 8), four for
    the last eight, each byte ceil(q * 256 / 243); the scale moves to the
    end."""
    code = lambda i: (block[2 + i // 4] >> (2 * (i % 4))) & 3
    out = bytearray(28)
    position = 0
    for width in (16, 8):
        start = position // 5
        for m in range(width):
            q = 0
            for n in range(5):
                q = q * 3 + code(position + m + n * width)
            out[start + m] = -(-q * 256 // 243)
        position += width * 5
    for h in range(2):
        q = 0
        for n in range(4):
            q = q * 3 + code(120 + h + n * 2)
        out[24 + h] = -(-q * 3 * 256 // 243)
    out[26:28] = block[0:2]
    return bytes(out)


def test_ptq_decoder_matches_native_codec_capture(cap):
    from oracle import oracle
    blocks = 0
    for c in cap["cases"]:
        pq2b = bytes.fromhex(c["pq2_hex"])
        ptqb = bytes.fromhex(c["ptq_hex"])
        n = c["rows"] * c["blocks_per_row"]
        assert len(pq2b) == 34 * n and len(ptqb) == 28 * n
        for i in range(n):
            a = pq2b[34 * i:34 * (i + 1)]
            b = ptqb[28 * i:28 * (i + 1)]
            assert np.array_equal(oracle.packed_values(143, np.frombuffer(b, np.uint8)),
                                  oracle.packed_values(142, np.frombuffer(a, np.uint8))), i
            assert b[26:28] == a[0:2]
            blocks += 1
    assert blocks == 992  # 169 rows of 2, 40, 48 or 136 blocks


def test_half_conversions_match_capture(cap):
    from oracle import oracle
    L = oracle.lib()
    for h, bits in cap["half_conversions"]:
        got = np.float32(L.po_half_to_float(h)).view(np.uint32)
        if np.isnan(np.float32(L.po_half_to_float(h))):
            assert (bits & 0x7F800000) == 0x7F800000 and (bits & 0x7FFFFF) != 0
        else:
            assert int(got) == bits, hex(h)


def test_pack_helper_reproduces_captured_ptq_bytes(cap):
    for c in cap["cases"][:40]:
        pq2b = bytes.fromhex(c["pq2_hex"])
        ptqb = bytes.fromhex(c["ptq_hex"])
        for i in range(c["rows"] * c["blocks_per_row"]):
            a = pq2b[34 * i:34 * (i + 1)]
            if any(byte & (byte >> 1) & 0x55 for byte in a[2:]):
                continue  # code 3 has no PTQ encoding
            assert pack_ptq(a) == ptqb[28 * i:28 * (i + 1)]


def mv(kind, blocks, cols, x, rows=1, fused=False):
    from oracle import oracle
    w = np.frombuffer(b"".join(blocks), np.uint8)
    return oracle.packed_matvec(kind, w, rows, cols, np.asarray(x, np.float32), fused)


def test_pq2_q8k_ties_even_and_per_half_scales():
    from oracle import oracle
    first = pq2(0x3C00, [(1, 2), (2, 2), (3, 2)])
    second = pq2(0x3800, [(0, 0)])
    x = np.zeros(256, np.float32)
    x[0], x[1], x[2], x[3], x[128], x[255] = 127.0, 0.5, 1.5, 2.5, -1.5, -127.0
    assert oracle.packed_uses_q8k(142, 256)
    assert mv(142, [first, second], 256, x).tolist() == [5.0]
    assert mv(142, [first, second], 256, x, fused=True).tolist() == [5.0]
    row = oracle.packed_row(142, np.frombuffer(first + second, np.uint8), 256, 0)
    assert float(np.sum((row * x).astype(np.float32), dtype=np.float32)) == 5.25


def test_pq2_code_three_zero_scale_and_zero_activations():
    from oracle import oracle
    first = pq2(0x3C00, [(0, 3)])
    second = pq2(0, [(0, 3)])
    row = oracle.packed_row(142, np.frombuffer(first + second, np.uint8), 256, 0)
    assert row[0] == 2.0 and row[128] == 0.0
    x = np.zeros(256, np.float32)
    x[0] = -127.0
    assert mv(142, [first, second], 256, x).tolist() == [-254.0]
    assert mv(142, [first, second], 256, np.zeros(256)).tolist() == [0.0]


def test_ptq1_q8_0_round_away_and_32_wide_scales():
    block = pack_ptq(pq2(0x4000, [(1, 2), (2, 2), (33, 2)]))
    x = np.zeros(128, np.float32)
    x[0], x[1], x[2], x[32], x[33] = 127.0, 0.5, 1.5, 63.5, 0.25
    assert mv(143, [block], 128, x).tolist() == [7.0]


def test_ptq1_activation_scales_are_rounded_to_fp16():
    block = pack_ptq(pq2(0x3C00, [(0, 2)]))
    x = np.zeros(128, np.float32)
    x[0] = 1.0
    assert mv(143, [block], 128, x).tolist() == [np.float32(0.99993896)]


def test_pq2_rows_off_256_take_the_q8_0_contract():
    from oracle import oracle
    first = pq2(0x4000, [(1, 2), (2, 3), (33, 2)])
    x = np.zeros(128, np.float32)
    x[0], x[1], x[2], x[32], x[33] = 127.0, 0.5, 1.5, 63.5, 0.25
    assert not oracle.packed_uses_q8k(142, 128)
    assert mv(142, [first], 128, x).tolist() == [11.0]
    second = pq2(0x3800, [(1, 2), (2, 3), (33, 2)])
    third = pq2(0x3C00, [(1, 2), (2, 3), (33, 2)])
    assert mv(142, [first, second, third], 384, np.concatenate([x, x, x])).tolist() == [19.25]


def test_ptq1_rows_equal_their_pq2_source():
    from oracle import oracle
    symbols = [(i, (i * 7 + i // 3) % 3) for i in range(128)]
    native = pq2(0x3555, symbols)
    packed = pack_ptq(native)
    a = oracle.packed_row(142, np.frombuffer(native, np.uint8), 128, 0)
    b = oracle.packed_row(143, np.frombuffer(packed, np.uint8), 128, 0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # the same matvec through both formats under the Q8_0 contract
    x = np.random.default_rng(3).standard_normal(128).astype(np.float32)
    assert mv(142, [native], 128, x).view(np.uint32).tolist() == \
        mv(143, [packed], 128, x).view(np.uint32).tolist()
