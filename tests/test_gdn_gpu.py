"""GPU Gated DeltaNet against the CPU oracle.

Decode: the reference's Source step (binary32 products summed in binary64),
compared within 2 ulp-scale bounds (the sums are reordered in binary64).
Chunked prefill (chunk 64, binary32 WY form): within the reference's
chunkwise bound 1e-3 + 1e-3*|ref| of the exact sequential recurrence
(reference docs/cpu-tiled-prefill.md:173-189).
"""
import numpy as np
import pytest
import torch

import prism_b200 as pb

pytestmark = pytest.mark.gpu


def inputs(batch, T, heads, key_heads, seed, d=128):
    """configs[2] inputs: q, k ~ N(0,1) L2-normalised per head; v ~ N(0,1);
    decay = exp(-softplus(N(0,1))); beta = sigmoid(N(0,1))."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((batch, T, key_heads, d)).astype(np.float32)
    k = rng.standard_normal((batch, T, key_heads, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((batch, T, heads, d)).astype(np.float32)
    decay = np.exp(-np.log1p(np.exp(rng.standard_normal((batch, T, heads))))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((batch, T, heads))))).astype(np.float32)
    return q, k, v, decay, beta


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def ex():
    e = pb.ProjectionExecutor(0)
    yield e
    e.close()


@pytest.mark.parametrize("batch", [1, 16, 64])
def test_decode_step_matches_oracle(ex, oracle, batch):
    heads, key_heads, d = 16, 16, 128
    q, k, v, decay, beta = inputs(batch, 1, heads, key_heads, seed=batch)
    state = (np.random.default_rng(99).standard_normal((batch, heads, d, d)) * 0.1).astype(np.float32)
    S, Q, K, V, G, B = map(dev, (state, q, k, v, decay, beta))
    O = torch.zeros((batch, 1, heads, d), device="cuda")
    pb.gdn_decode_device(ex, batch, heads, key_heads, S.data_ptr(), Q.data_ptr(), K.data_ptr(),
                         V.data_ptr(), G.data_ptr(), B.data_ptr(), O.data_ptr())
    torch.cuda.synchronize()
    ex.sync()
    Sg, Og = S.cpu().numpy(), O.cpu().numpy()
    for b in sorted({0, batch // 2, batch - 1}):
        for h in (0, 7, 15):
            nxt, out = oracle.gdn_head_step(state[b, h], q[b, 0, h % key_heads], k[b, 0, h % key_heads],
                                            v[b, 0, h], float(decay[b, 0, h]), float(beta[b, 0, h]))
            assert np.allclose(Sg[b, h], nxt, rtol=1e-6, atol=1e-7)
            assert np.allclose(Og[b, 0, h], out, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("T,chunk,key_heads", [(200, 64, 4), (300, 37, 2), (64, 64, 4), (5, 64, 4)])
def test_chunked_prefill_within_chunkwise_bound(ex, oracle, T, chunk, key_heads):
    batch, heads, d = 2, 4, 128
    q, k, v, decay, beta = inputs(batch, T, heads, key_heads, seed=T)
    state = (np.random.default_rng(7).standard_normal((batch, heads, d, d)) * 0.1).astype(np.float32)
    S, Q, K, V, G, B = map(dev, (state, q, k, v, decay, beta))
    O = torch.zeros((batch, T, heads, d), device="cuda")
    pb.gdn_prefill_device(ex, batch, T, heads, key_heads, chunk, S.data_ptr(), Q.data_ptr(),
                          K.data_ptr(), V.data_ptr(), G.data_ptr(), B.data_ptr(), O.data_ptr())
    torch.cuda.synchronize()
    ex.sync()
    Sg, Og = S.cpu().numpy(), O.cpu().numpy()
    for b in range(batch):
        for h in range(heads):
            kh = h % key_heads
            se, oe = oracle.gdn_head_prefill(state[b, h], q[b, :, kh], k[b, :, kh], v[b, :, h],
                                             decay[b, :, h], beta[b, :, h])
            assert np.all(np.abs(Og[b, :, h] - oe) <= 1e-3 + 1e-3 * np.abs(oe)), (b, h)
            assert np.all(np.abs(Sg[b, h] - se) <= 1e-3 + 1e-3 * np.abs(se)), (b, h)


def test_config2_prefill_4096_tokens(ex, oracle):
    """configs[2] prefill geometry: 16 heads, T = 4096, chunk 64, B = 1;
    four heads checked against the exact sequential recurrence."""
    batch, T, heads, d = 1, 4096, 16, 128
    q, k, v, decay, beta = inputs(batch, T, heads, heads, seed=4096)
    state = np.zeros((batch, heads, d, d), np.float32)
    S, Q, K, V, G, B = map(dev, (state, q, k, v, decay, beta))
    O = torch.zeros((batch, T, heads, d), device="cuda")
    pb.gdn_prefill_device(ex, batch, T, heads, heads, 64, S.data_ptr(), Q.data_ptr(),
                          K.data_ptr(), V.data_ptr(), G.data_ptr(), B.data_ptr(), O.data_ptr())
    torch.cuda.synchronize()
    ex.sync()
    Sg, Og = S.cpu().numpy(), O.cpu().numpy()
    for h in (0, 5, 10, 15):
        se, oe = oracle.gdn_head_prefill(state[0, h], q[0, :, h], k[0, :, h], v[0, :, h],
                                         decay[0, :, h], beta[0, :, h])
        assert np.all(np.abs(Og[0, :, h] - oe) <= 1e-3 + 1e-3 * np.abs(oe)), h
        assert np.all(np.abs(Sg[0, h] - se) <= 1e-3 + 1e-3 * np.abs(se)), h


def test_prefill_is_batch_invariant(ex):
    """A sequence prefilled alone and as row 5 of a batch of 16 gives the
    same bits: every output keeps one accumulation order whatever the grid,
    and each (sequence, head) reads only its own chunk scratch.  The nonzero
    starting state and a ragged last chunk cover the state update and the
    zero-filled rows."""
    T, heads, d = 1000, 16, 128
    q, k, v, decay, beta = inputs(16, T, heads, heads, seed=77)
    rng = np.random.default_rng(78)
    state = (rng.standard_normal((16, heads, d, d)) * 0.1).astype(np.float32)
    outs = {}
    for batch in (1, 16):
        sl = slice(5, 6) if batch == 1 else slice(0, 16)
        S, Q, K, V, G, B = map(dev, (state[sl], q[sl], k[sl], v[sl], decay[sl], beta[sl]))
        O = torch.zeros((batch, T, heads, d), device="cuda")
        pb.gdn_prefill_device(ex, batch, T, heads, heads, 64, S.data_ptr(), Q.data_ptr(),
                              K.data_ptr(), V.data_ptr(), G.data_ptr(), B.data_ptr(),
                              O.data_ptr())
        torch.cuda.synchronize()
        ex.sync()
        i = 0 if batch == 1 else 5
        outs[batch] = (S.cpu().numpy()[i], O.cpu().numpy()[i])
    for a, b in zip(outs[1], outs[16]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
