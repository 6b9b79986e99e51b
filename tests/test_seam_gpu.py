"""The rest of the executor trait through the C ABI: capacity and
eligibility queries, sibling projections over token tiles, the fused
gate/up + SwiGLU (one token and a tile) and the single-token FFN chain.

Every output must equal, bit for bit, what the executor's per-token group
projection (prism_b200_project_f32_group, itself bit-exact against the
oracle in test_projection_gpu.py) and the binary32 SwiGLU give for the same
token; the FFN chain is also compared with the oracle's chain and with the
token-tile chain.  Unsupported requests (Q8_0 activations for these kinds,
a Hadamard-rotated chain) are refused before any submission and leave the
executor open, as the reference's eligibility rules require.
"""
import numpy as np
import pytest

import prism_b200 as pb
import synth

pytestmark = pytest.mark.gpu

H, F = 512, 1024


def swiglu(up, gate):
    """up * silu(gate) in binary32, exp evaluated in binary64 and rounded
    once (the kernels' and the oracle's transcendental)."""
    g = np.asarray(gate, np.float32)
    e = np.exp(-g.astype(np.float64)).astype(np.float32)
    return (np.asarray(up, np.float32) * (g / (np.float32(1.0) + e))).astype(np.float32)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def ex():
    with pb.ProjectionExecutor(0) as e:
        yield e


@pytest.mark.parametrize("kind", [pb.KIND_TQ2_0, pb.KIND_Q2_K])
def test_capacity_and_eligibility(ex, kind):
    gen = synth.tq2_weights if kind == pb.KIND_TQ2_0 else synth.q2k_weights
    gate = pb.Tensor(kind, H, F, gen(F, H, 1))
    up = pb.Tensor(kind, H, F, gen(F, H, 2))
    down = pb.Tensor(kind, F, H, gen(H, F, 3))
    odd = pb.Tensor(kind, H, F // 2, gen(F // 2, H, 4))
    assert ex.operation_capacity() is None
    assert ex.supports_f32(gate) and ex.supports_tile_tokens()
    assert ex.supports_f32_group([gate, up]) and not ex.supports_f32_group([gate, down])
    assert not ex.supports_q8(gate)
    assert ex.supports_f32_ffn_swiglu(gate, up) and not ex.supports_f32_ffn_swiglu(gate, odd)
    assert ex.supports_f32_ffn_chain(gate, up, down)
    assert not ex.supports_f32_ffn_chain(gate, up, gate)
    # Q8_0 activations are refused before submission; the executor stays open
    with pytest.raises(pb.PrismB200Error):
        ex.project_q8(gate, np.zeros(H // 32 * 34, np.uint8))
    x = synth.activations(H, 5)
    assert ex.project_f32(gate, x).shape == (F,)


@pytest.mark.parametrize("kind", [pb.KIND_TQ2_0, pb.KIND_Q2_K])
@pytest.mark.parametrize("tokens", [1, 7, 130])
def test_pair_and_triple_tokens_match_group(ex, kind, tokens):
    gen = synth.tq2_weights if kind == pb.KIND_TQ2_0 else synth.q2k_weights
    ws = [pb.Tensor(kind, H, rows, gen(rows, H, 10 + i)) for i, rows in enumerate((F, 256, 768))]
    x = np.random.default_rng(tokens).standard_normal((tokens, H)).astype(np.float32)
    a, b = ex.project_f32_pair_tokens(ws[:2], x)
    c3 = ex.project_f32_triple_tokens(ws, x)
    for t in list(range(min(tokens, 4))) + [tokens - 1]:
        ref = ex.project_f32_group(ws, x[t])
        assert np.array_equal(bits(a[t]), bits(ref[0])), t
        assert np.array_equal(bits(b[t]), bits(ref[1])), t
        for k in range(3):
            assert np.array_equal(bits(c3[k][t]), bits(ref[k])), (t, k)


@pytest.mark.parametrize("kind", [pb.KIND_TQ2_0, pb.KIND_Q2_K])
def test_ffn_swiglu_one_token_and_tile(ex, kind):
    gen = synth.tq2_weights if kind == pb.KIND_TQ2_0 else synth.q2k_weights
    gate = pb.Tensor(kind, H, F, gen(F, H, 21))
    up = pb.Tensor(kind, H, F, gen(F, H, 22))
    x = np.random.default_rng(23).standard_normal((9, H)).astype(np.float32)
    tile = ex.project_f32_ffn_swiglu_tokens(gate, up, x)
    for t in range(x.shape[0]):
        one = ex.project_f32_ffn_swiglu(gate, up, x[t])
        g, u = ex.project_f32_group([gate, up], x[t])
        ref = swiglu(u, g)
        assert np.array_equal(bits(one), bits(ref)), t
        assert np.array_equal(bits(tile[t]), bits(ref)), t


@pytest.mark.parametrize("kind", [pb.KIND_TQ2_0, pb.KIND_Q2_K])
def test_ffn_chain_one_token(ex, kind):
    from oracle import oracle
    gen = synth.tq2_weights if kind == pb.KIND_TQ2_0 else synth.q2k_weights
    wg, wu, wd = gen(F, H, 31), gen(F, H, 32), gen(H, F, 33)
    gate, up, down = pb.Tensor(kind, H, F, wg), pb.Tensor(kind, H, F, wu), pb.Tensor(kind, F, H, wd)
    rng = np.random.default_rng(34)
    ffn = pb.FfnChain(ex, gate, up, down, max_tokens=4)
    try:
        for t in range(4):
            x = rng.standard_normal(H).astype(np.float32)
            res = rng.standard_normal(H).astype(np.float32) if t % 2 else None
            out = ex.project_f32_ffn_chain(gate, up, down, x, residual=res)
            # the oracle's chain: Q8_K(x) -> gate, up -> SwiGLU -> Q8_K -> down (+ residual)
            act = oracle.q8k_quantize(x)
            g = oracle.matvec(kind, wg, F, H, act)
            u = oracle.matvec(kind, wu, F, H, act)
            y = oracle.matvec(kind, wd, H, F, oracle.q8k_quantize(swiglu(u, g)))
            if res is not None:
                y = (res + y).astype(np.float32)
            assert np.array_equal(bits(out), bits(y)), t
            tile = ffn(x[None, :], None if res is None else res[None, :])
            assert np.array_equal(bits(out), bits(tile[0])), t
    finally:
        ffn.close()
    # a rotated chain is refused before submission; the executor stays open
    with pytest.raises(pb.PrismB200Error):
        ex.project_f32_ffn_chain(gate, up, down, np.ones(H, np.float32), hadamard_block_size=64)
    assert ex.project_f32(gate, np.ones(H, np.float32)).shape == (F,)
