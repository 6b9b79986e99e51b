"""Multi-token projection (prefill GEMM, configs[3]) against the CPU oracle.

prism_b200_project_f32_tokens quantizes every token to Q8_K and runs the
integer block dots on the tensor cores; each output must equal, bit for bit,
the oracle's per-token dot (reference src/kernels/prefill.rs:48-87) and the
single-token projection prism_b200_project_f32.
"""
import numpy as np
import pytest
import torch

import prism_b200 as pb
import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ex():
    e = pb.ProjectionExecutor(0)
    yield e
    e.close()


def weights(kind, rows, cols, seed):
    return synth.tq2_weights(rows, cols, seed) if kind == 35 else synth.q2k_weights(rows, cols, seed)


def tokens(M, cols, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((M, cols)) * scale).astype(np.float32)


def same_bits(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32),
                          np.ascontiguousarray(b).view(np.uint32))


@pytest.mark.parametrize("kind", [35, 10])
@pytest.mark.parametrize("M,rows,cols", [(1, 128, 256), (5, 200, 2560), (128, 128, 512),
                                         (130, 300, 2560), (300, 1000, 9216), (33, 77, 768)])
def test_tokens_bit_exact(ex, oracle, kind, M, rows, cols):
    seed = M * 31 + rows + cols
    w = weights(kind, rows, cols, seed)
    x = tokens(M, cols, seed + 1)
    t = pb.Tensor(kind, cols, rows, w)
    y = ex.project_f32_tokens(t, x)
    y_ref = oracle.project_tokens(kind, w, rows, cols, x, threads=8)
    assert same_bits(y, y_ref)
    # the same token through the single-token projection
    for m in sorted({0, M - 1}):
        assert same_bits(ex.project_f32(t, x[m]), y_ref[m])


@pytest.mark.parametrize("kind", [35, 10])
def test_pinned_and_wide_range(ex, oracle, kind):
    rows, cols = 260, 2560
    w = weights(kind, rows, cols, 5)
    x = np.concatenate([tokens(40, cols, 6, 1e-3), tokens(40, cols, 7, 1e3),
                        np.zeros((3, cols), np.float32)])
    t = pb.Tensor(kind, cols, rows, w)
    for pinned in (False, True):
        y = ex.project_f32_tokens(t, x, pinned=pinned)
        assert same_bits(y, oracle.project_tokens(kind, w, rows, cols, x, pinned, threads=8))
    # an all-zero token projects to +0.0 everywhere
    assert same_bits(y[-1], np.zeros(rows, np.float32))


@pytest.mark.parametrize("kind", [35, 10])
@pytest.mark.parametrize("cols,rows", [(2560, 9216), (9216, 2560)])
def test_config3_shapes_sampled_tokens(ex, oracle, kind, cols, rows):
    """2048 tokens at both FFN shapes; a sample of tokens is
    recomputed by the oracle (each token's outputs depend on that token only)."""
    M = 2048
    w = weights(kind, rows, cols, 3)
    x = tokens(M, cols, 4)
    t = pb.Tensor(kind, cols, rows, w)
    wt = ex.upload(t)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((M, rows), device="cuda")
    ex.project_f32_tokens_device(wt, M, xd.data_ptr(), yd.data_ptr())
    ex.sync()
    y = yd.cpu().numpy()
    assert np.isfinite(y).all()
    sample = [0, 1, 127, 128, 1000, 1535, 2046, 2047]
    y_ref = oracle.project_tokens(kind, w, rows, cols, x[sample], threads=16)
    assert same_bits(y[sample], y_ref)


def test_errors(ex):
    rows, cols = 64, 512
    w = weights(35, rows, cols, 9)
    t = pb.Tensor(35, cols, rows, w)
    wt = ex.upload(t)
    # no tokens: nothing to do
    ex.project_f32_tokens_device(wt, 0, 0, 0)
    with pytest.raises(pb.PrismB200Error) as err:
        ex.project_f32_tokens(t, np.zeros((3, 256), np.float32))
    assert err.value.code == pb.E_INVALID
    x = torch.zeros((2, cols), device="cuda")
    y = torch.zeros((2, rows), device="cuda")
    with pytest.raises(pb.PrismB200Error) as err:
        ex.project_f32_tokens_device(wt, 1 << 17, x.data_ptr(), y.data_ptr())
    assert err.value.code == pb.E_INVALID
    with pytest.raises(pb.PrismB200Error) as err:
        ex.project_f32_tokens_device(wt, 2, x.data_ptr() + 4, y.data_ptr())
    assert err.value.code == pb.E_INVALID
    # nonfinite activations are reported, outputs zeroed, executor faulted
    bad = np.ones((2, cols), np.float32)
    bad[1, 7] = np.inf
    with pytest.raises(pb.PrismB200Error) as err:
        ex.project_f32_tokens(t, bad)
    assert err.value.code == pb.E_NONFINITE
    ex.reset()
    assert np.isfinite(ex.project_f32_tokens(t, np.ones((2, cols), np.float32))).all()
