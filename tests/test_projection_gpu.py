"""GPU parity of the packed projection path against the CPU oracle.

Integer block dots and Q8_K bytes are compared bit for bit; projection
outputs are compared bit for bit as well (the kernels keep the reference's
sequential binary32 chain), which is stricter than the 1e-5 relative bound
the benchmark configuration states.
"""
import json
import os

import numpy as np
import pytest

import prism_b200 as pb
import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ex():
    e = pb.ProjectionExecutor(0)
    yield e
    e.close()


def _golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("name,kind", [("tq2_0.json", 35), ("q2_k.json", 10)])
def test_golden_generic_dot(ex, name, kind):
    for case in _golden(name):
        packed = np.frombuffer(bytes.fromhex(case["OutputHex"]), np.uint8)
        act = np.frombuffer(bytes.fromhex(case["ActivationsHex"]), pb.Q8K_DTYPE)
        t = pb.Tensor(kind, case["Count"], 1, packed.copy(), case["Name"])
        y = ex.project(t, act)
        assert y.tobytes().hex() == case["GenericDotHex"], case["Name"]


@pytest.mark.parametrize("kind", [35, 10])
@pytest.mark.parametrize("rows,cols", [(1, 256), (7, 512), (33, 2560), (100, 9216), (4096, 4096),
                                       (2560, 9216), (9500, 512), (10000, 16384)])
def test_block_dots_and_projection_bit_exact(ex, oracle, kind, rows, cols):
    seed = rows * 7 + cols
    w = synth.tq2_weights(rows, cols, seed) if kind == 35 else synth.q2k_weights(rows, cols, seed)
    x = synth.activations(cols, seed + 1)
    act = oracle.q8k_quantize(x)
    t = pb.Tensor(kind, cols, rows, w)
    y = ex.project(t, act)
    y_ref = oracle.matvec(kind, w, rows, cols, act, threads=8)
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    dots = ex.block_dots(t, act)
    for r in sorted({0, rows // 2, rows - 1}):
        ref = oracle.block_dots(kind, w[r], act)
        if kind == 35:
            assert np.array_equal(dots[r], ref)
        else:
            assert np.array_equal(dots[0][r], ref[0]) and np.array_equal(dots[1][r], ref[1])


def test_q8k_quantize_bit_exact(ex, oracle):
    rng = np.random.default_rng(11)
    cases = [
        rng.standard_normal(4096).astype(np.float32),
        np.zeros(256, np.float32),
        (rng.standard_normal(2560) * 1e-30).astype(np.float32),
        (rng.standard_normal(9216) * 1e4).astype(np.float32),
    ]
    ties = np.zeros(256, np.float32)
    ties[0], ties[255], ties[1], ties[2], ties[3] = 127.0, -127.0, 0.5, 1.5, 2.5
    cases.append(ties)
    neg_first = np.zeros(256, np.float32)
    neg_first[3], neg_first[200] = -2.0, 2.0
    cases.append(neg_first)
    for x in cases:
        for pinned in (False, True):
            got = ex.quantize_q8k(x, pinned=pinned)
            ref = oracle.q8k_quantize(x, pinned=pinned)
            assert got.tobytes() == ref.tobytes()


def test_q8k_pinned_golden_block(ex):
    with open(os.path.join(GOLDEN, "q8k_parity.json")) as f:
        cases = json.load(f)["cases"]
    for c in cases:
        x = np.zeros(256, np.float32)
        x[0] = np.frombuffer(bytes.fromhex(c["input_bits"][0]), ">f4")[0]
        x[1] = np.frombuffer(bytes.fromhex(c["input_bits"][1]), ">f4")[0]
        assert ex.quantize_q8k(x, pinned=True).tobytes().hex() == c["native_block_hex"]
        assert int(ex.quantize_q8k(x)["values"][0][1]) == c["source_code_at_1"]


def test_project_f32_and_group(ex, oracle):
    cols = 2560
    ws = [synth.tq2_weights(r, cols, 100 + r) for r in (6144, 2048, 16, 16)]
    ts = [pb.Tensor(35, cols, w.shape[0], w) for w in ws]
    x = synth.activations(cols, 5)
    act = oracle.q8k_quantize(x)
    outs = ex.project_f32_group(ts, x)
    for t, w, y in zip(ts, ws, outs):
        ref = oracle.matvec(35, w, t.rows, cols, act, threads=8)
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
    y1 = ex.project_f32(ts[1], x)
    assert np.array_equal(y1, outs[1])


def test_eligibility_and_operation_count(ex):
    z = np.zeros(1, np.uint8)
    assert ex.supports(pb.Tensor(35, 2560, 9216, z))
    assert ex.supports(pb.Tensor(10, 9216, 2560, z))
    assert not ex.supports(pb.Tensor(35, 2500, 10, z))
    # the reference's own PQ2 / PTQ1 formats: whole 128-weight blocks
    assert ex.supports(pb.Tensor(142, 256, 10, z)) and ex.supports(pb.Tensor(143, 384, 10, z))
    assert not ex.supports(pb.Tensor(142, 200, 10, z))
    # TQ1_0 and Q3_K..Q6_K: whole 256-weight blocks, one unit per row and block
    for kind in (34, 11, 12, 13, 14):
        assert ex.supports(pb.Tensor(kind, 512, 10, z))
        assert not ex.supports(pb.Tensor(kind, 384, 10, z))
        assert ex.operation_count(pb.Tensor(kind, 512, 10, z)) == 20
    # units of (tile of H rows) x (256-column block); H is 8, 16 or 32
    n = ex.operation_count(pb.Tensor(35, 4096, 4096, z))
    assert n in (512 * 16, 256 * 16, 128 * 16)
    assert ex.operation_count(pb.Tensor(15, 256, 1, z)) is None  # Q8_K is an activation


def test_errors_are_terminal_and_clear_output(oracle):
    with pb.ProjectionExecutor(0) as ex:
        w = synth.tq2_weights(64, 512, 3)
        bad = w.copy()
        bad[5, 64:66] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
        with pytest.raises(pb.PrismB200Error) as e:
            ex.upload(pb.Tensor(35, 512, 64, bad))
        assert e.value.code == pb.E_NONFINITE
        with pytest.raises(pb.PrismB200Error) as e:
            ex.upload(pb.Tensor(35, 500, 64, w))
        assert e.value.code == pb.E_UNSUPPORTED
        t = pb.Tensor(35, 512, 64, w)
        wt = ex.upload(t)
        act = oracle.q8k_quantize(synth.activations(512, 4))
        good = ex.project(wt, act)
        act_bad = act.copy()
        act_bad["scale"][1] = np.float32(np.nan)
        with pytest.raises(pb.PrismB200Error) as e:
            ex.project(wt, act_bad)
        assert e.value.code == pb.E_NONFINITE
        # the executor is closed until reset; no CPU replay happened
        with pytest.raises(pb.PrismB200Error) as e:
            ex.project(wt, act)
        assert e.value.code == pb.E_FAULTED
        ex.reset()
        assert np.array_equal(ex.project(wt, act), good)
        # nonfinite f32 activations are rejected by the quantizer
        x = synth.activations(512, 9)
        x[7] = np.inf
        with pytest.raises(pb.PrismB200Error) as e:
            ex.project_f32(wt, x)
        assert e.value.code == pb.E_NONFINITE
        ex.reset()
