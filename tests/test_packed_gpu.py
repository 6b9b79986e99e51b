"""PQ2 (type 142) and PTQ1 (type 143) projections through the C ABI against
the oracle, bit for bit.

  * project_f32 under both activation contracts: PQ2 with a multiple of 256
    columns (Q8_K), PQ2 with an odd 128-block count and PTQ1 (Q8_0), at
    configs[1] widths and odd shapes, codes 0-3 and PTQ1's every byte;
  * project (prepared Q8_K blocks, fused and unfused) and project_q8
    (prepared Q8_0 blocks) against the oracle's per-row dots;
  * the reference's known answers (reference tests/kernels.rs:206-320)
    through the device;
  * refusals that leave the executor open: a contract mismatch, pinned
    accumulation, and every tiled-only path given a packed weight.
"""
import numpy as np
import pytest

import prism_b200 as pb

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def rand_packed(kind, rows, cols, seed, code3=True):
    """Random rows of `kind`: PQ2 codes 0..3 (or 0..2), PTQ1 any byte, both
    with finite binary16 scales of either sign."""
    rng = np.random.default_rng(seed)
    nb = cols // 128
    bb = pb.PACKED_BLOCK_BYTES[kind]
    blocks = rng.integers(0, 256, size=(rows * nb, bb), dtype=np.uint8)
    if kind == pb.KIND_PQ2 and not code3:
        c = blocks[:, 2:]
        c &= ~((c & (c >> 1) & 0x55) << 1) & 0xFF  # code 3 -> code 1
    scales = (rng.uniform(0.02, 0.2, rows * nb) * rng.choice([-1, 1], rows * nb)).astype(np.float16)
    at = 0 if kind == pb.KIND_PQ2 else 26
    blocks[:, at:at + 2] = scales.view(np.uint8).reshape(-1, 2)
    return blocks.reshape(rows, nb * bb)


def q8_blocks(x):
    """The oracle's Q8_0 activation blocks in the ABI layout."""
    from oracle import oracle
    q = oracle.q8_0_quantize(x)
    out = np.zeros(q.size, pb.Q8_DTYPE)
    out["scale"] = np.array([oracle.lib().po_half_to_float(int(d)) for d in q["d"]], np.float32)
    out["values"] = q["values"]
    return out


@pytest.fixture(scope="module")
def ex():
    with pb.ProjectionExecutor(0) as e:
        yield e


@pytest.mark.parametrize("kind,rows,cols", [
    (pb.KIND_PQ2, 2560, 2560),     # Q8_K contract, configs[1] width
    (pb.KIND_PQ2, 97, 9216),
    (pb.KIND_PQ2, 130, 384),       # odd 128-block count: Q8_0 contract
    (pb.KIND_PTQ1, 2560, 2560),
    (pb.KIND_PTQ1, 33, 128),
    (pb.KIND_PTQ1, 300, 4480),     # 35 blocks: more than one round of 32
])
def test_project_f32_matches_oracle(ex, kind, rows, cols):
    from oracle import oracle
    w = rand_packed(kind, rows, cols, seed=rows + cols)
    t = pb.Tensor(kind, cols, rows, w)
    assert ex.supports(t) and ex.operation_count(t) == rows * (cols // 128)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    got = ex.project_f32(t, x)
    want = oracle.packed_matvec(kind, w, rows, cols, x)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("fused", [False, True])
def test_project_prepared_q8k_blocks(ex, fused):
    from oracle import oracle
    rows, cols = 200, 2560
    w = rand_packed(pb.KIND_PQ2, rows, cols, seed=7)
    t = pb.Tensor(pb.KIND_PQ2, cols, rows, w)
    x = np.random.default_rng(8).standard_normal(cols).astype(np.float32)
    act = oracle.q8k_quantize(x)
    got = ex.project(t, act, fused=fused)
    want = np.array([oracle.pq2_dot_q8k(w[r], act, fused) for r in range(rows)], np.float32)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("kind", [pb.KIND_PQ2, pb.KIND_PTQ1])
def test_project_q8_prepared_blocks(ex, kind):
    from oracle import oracle
    rows, cols = 150, 1152
    w = rand_packed(kind, rows, cols, seed=11)
    t = pb.Tensor(kind, cols, rows, w)
    x = np.random.default_rng(12).standard_normal(cols).astype(np.float32)
    act = q8_blocks(x)
    got = ex.project_q8(t, act)
    want = np.array([oracle.packed_dot_q8(kind, w[r], oracle.q8_0_quantize(x))
                     for r in range(rows)], np.float32)
    assert np.array_equal(bits(got), bits(want))


def pq2(scale, symbols):
    b = bytearray([0x55] * 34)
    b[0:2] = int(scale).to_bytes(2, "little")
    for index, symbol in symbols:
        shift = 2 * (index % 4)
        b[2 + index // 4] &= ~(3 << shift) & 0xFF
        b[2 + index // 4] |= symbol << shift
    return bytes(b)


def test_reference_known_answers(ex):
    from test_oracle_packed import pack_ptq
    def run(kind, blocks, cols, x):
        t = pb.Tensor(kind, cols, 1, np.frombuffer(b"".join(blocks), np.uint8).reshape(1, -1))
        return ex.project_f32(t, np.asarray(x, np.float32)).tolist()
    x = np.zeros(256, np.float32)
    x[0], x[1], x[2], x[3], x[128], x[255] = 127.0, 0.5, 1.5, 2.5, -1.5, -127.0
    assert run(142, [pq2(0x3C00, [(1, 2), (2, 2), (3, 2)]), pq2(0x3800, [(0, 0)])], 256, x) == [5.0]
    x = np.zeros(256, np.float32)
    x[0] = -127.0
    assert run(142, [pq2(0x3C00, [(0, 3)]), pq2(0, [(0, 3)])], 256, x) == [-254.0]
    x = np.zeros(128, np.float32)
    x[0], x[1], x[2], x[32], x[33] = 127.0, 0.5, 1.5, 63.5, 0.25
    assert run(143, [pack_ptq(pq2(0x4000, [(1, 2), (2, 2), (33, 2)]))], 128, x) == [7.0]
    first = pq2(0x4000, [(1, 2), (2, 3), (33, 2)])
    assert run(142, [first], 128, x) == [11.0]
    three = [first, pq2(0x3800, [(1, 2), (2, 3), (33, 2)]), pq2(0x3C00, [(1, 2), (2, 3), (33, 2)])]
    assert run(142, three, 384, np.concatenate([x, x, x])) == [19.25]
    x = np.zeros(128, np.float32)
    x[0] = 1.0
    assert run(143, [pack_ptq(pq2(0x3C00, [(0, 2)]))], 128, x) == [np.float32(0.99993896)]


def test_refusals_leave_the_executor_open(ex):
    from oracle import oracle
    w = rand_packed(pb.KIND_PTQ1, 64, 256, seed=21)
    t = pb.Tensor(pb.KIND_PTQ1, 256, 64, w)
    x = np.random.default_rng(22).standard_normal(256).astype(np.float32)
    with pytest.raises(pb.PrismB200Error) as e:   # PTQ1 takes Q8_0, not Q8_K
        ex.project(t, oracle.q8k_quantize(x))
    assert e.value.code == pb.E_UNSUPPORTED
    with pytest.raises(pb.PrismB200Error):
        ex.project_q8(t, q8_blocks(x), pinned=True)
    with pytest.raises(pb.PrismB200Error) as e:   # tiled-only paths
        ex.project_f32_group([t, t], x)
    assert e.value.code == pb.E_UNSUPPORTED
    assert not ex.supports_f32_group([t, t])
    assert ex.supports_q8(t) and ex.supports_f32(t)
    tq = pb.Tensor(pb.KIND_TQ2_0, 256, 64, pb.synth_weights(35, 64, 256, 3))
    assert not ex.supports_q8(tq)
    # still open: a valid projection runs
    assert np.array_equal(bits(ex.project_f32(t, x)),
                          bits(oracle.packed_matvec(pb.KIND_PTQ1, w, 64, 256, x)))
