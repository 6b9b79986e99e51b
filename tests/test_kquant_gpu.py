"""TQ1_0 (34) and Q3_K..Q6_K (11-14), the rest of the reference's Q8_K
activation contract (reference src/kernels.rs:1653-1674), through the C ABI
against the oracle, bit for bit:

  * the upstream golden vectors (tests/golden/{tq1_0,q3_k,q4_k,q5_k,q6_k}.json,
    from the reference's tests/fixtures/upstream-*quants.json): every case's
    packed row with its captured Q8_K activations gives the captured
    generic dot;
  * random rows at model widths through project (prepared Q8_K blocks) and
    project_f32 against oracle.matvec;
  * eligibility, operation counts and the refusals of the Q8_0 and tiled-only
    paths.
"""
import json
import os

import numpy as np
import pytest

import prism_b200 as pb

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = {34: "tq1_0.json", 11: "q3_k.json", 12: "q4_k.json", 13: "q5_k.json", 14: "q6_k.json"}
SCALES = {34: (52,), 11: (108,), 12: (0, 2), 13: (0, 2), 14: (208,)}


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def rand_rows(kind, rows, cols, seed):
    """Random blocks of `kind` with finite binary16 scales in a modest range."""
    rng = np.random.default_rng(seed)
    bb = pb.KQUANT_BLOCK_BYTES[kind]
    nb = rows * (cols // 256)
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    for off in SCALES[kind]:
        sc = rng.uniform(1e-3, 2e-2, nb).astype(np.float16)
        blk[:, off:off + 2] = sc.view(np.uint8).reshape(-1, 2)
    return blk.reshape(rows, -1)


@pytest.fixture(scope="module")
def ex():
    with pb.ProjectionExecutor(0) as e:
        yield e


@pytest.mark.parametrize("kind", [34, 11, 12, 13, 14])
def test_upstream_golden_dots_on_device(ex, kind):
    with open(os.path.join(GOLDEN, NAMES[kind])) as f:
        cases = json.load(f)["cases"]
    assert len(cases) == 5
    for c in cases:
        w = np.frombuffer(bytes.fromhex(c["OutputHex"]), np.uint8)
        act = np.frombuffer(bytes.fromhex(c["ActivationsHex"]), pb.Q8K_DTYPE)
        cols = act.size * 256
        t = pb.Tensor(kind, cols, 1, w.reshape(1, -1))
        assert ex.supports(t)
        got = ex.project(t, act)
        assert np.float32(got[0]).tobytes().hex() == c["GenericDotHex"], c["Name"]


@pytest.mark.parametrize("kind", [34, 11, 12, 13, 14])
@pytest.mark.parametrize("rows,cols", [(2560, 2560), (97, 9216), (33, 256)])
def test_random_rows_match_oracle(ex, kind, rows, cols):
    from oracle import oracle
    w = rand_rows(kind, rows, cols, seed=kind * 7 + rows)
    t = pb.Tensor(kind, cols, rows, w)
    assert ex.operation_count(t) == rows * (cols // 256)
    x = np.random.default_rng(cols + kind).standard_normal(cols).astype(np.float32)
    act = oracle.q8k_quantize(x)
    want = oracle.matvec(kind, w, rows, cols, act, threads=8)
    assert np.array_equal(bits(ex.project(t, act)), bits(want))
    assert np.array_equal(bits(ex.project_f32(t, x)), bits(want))


def test_refusals_leave_the_executor_open(ex):
    from oracle import oracle
    w = rand_rows(12, 64, 512, seed=3)
    t = pb.Tensor(12, 512, 64, w)
    x = np.random.default_rng(4).standard_normal(512).astype(np.float32)
    assert not ex.supports_q8(t)
    with pytest.raises(pb.PrismB200Error) as e:   # Q8_0 activations: PQ2/PTQ1 only
        ex.project_q8(t, np.zeros(16, pb.Q8_DTYPE))
    assert e.value.code == pb.E_UNSUPPORTED
    with pytest.raises(pb.PrismB200Error) as e:   # tiled-only paths
        ex.project_f32_group([t, t], x)
    assert e.value.code == pb.E_UNSUPPORTED
    assert not ex.supports(pb.Tensor(12, 384, 4, rand_rows(12, 4, 256, 1)))  # cols % 256
    got = ex.project_f32(t, x)
    assert np.array_equal(bits(got), bits(oracle.matvec(12, w, 64, 512, oracle.q8k_quantize(x))))


@pytest.mark.parametrize("kind,name", [(35, "tq2_0.json"), (34, "tq1_0.json")])
def test_tq_quantizer_on_device(ex, kind, name):
    """f32 -> TQ1_0 / TQ2_0 (reference src/kernels/tquants.rs:288-336): the
    golden InputHex -> OutputHex cases, random rows, a zero block, ties at
    +-0.5 * d, and the refusals."""
    from oracle import oracle
    with open(os.path.join(GOLDEN, name)) as f:
        cases = [c for c in json.load(f)["cases"] if "InputHex" in c]
    for c in cases:
        x = np.frombuffer(bytes.fromhex(c["InputHex"]), "<f4")
        assert ex.quantize_tq(kind, x).tobytes().hex() == c["OutputHex"], c["Name"]
    rng = np.random.default_rng(kind)
    x = (rng.standard_normal(256 * 40) * rng.uniform(1e-3, 10, 256 * 40)).astype(np.float32)
    x[:256] = 0.0                                  # a zero block
    x[256:512] = np.tile([1.0, 0.5, -0.5, 0.25], 64)  # exact ties at d / 2
    assert np.array_equal(ex.quantize_tq(kind, x), oracle.tq_quantize(kind, x))
    with pytest.raises(pb.PrismB200Error) as e:   # not a whole block
        ex.quantize_tq(kind, x[:300])
    assert e.value.code == pb.E_INVALID
    bad = x[:512].copy()
    bad[7] = np.inf
    with pytest.raises(pb.PrismB200Error) as e:
        ex.quantize_tq(kind, bad)
    assert e.value.code == pb.E_INVALID
    ex.reset()
    assert np.array_equal(ex.quantize_tq(kind, x[:512]), oracle.tq_quantize(kind, x[:512]))
