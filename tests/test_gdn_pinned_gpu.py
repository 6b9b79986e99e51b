"""The reference's pinned ("Swift") GDN recurrence on the device
(prism_b200_gdn_prefill_pinned_device; reference src/kernels/pinned_gdn.rs:
370-455 step_row_in_place over tokens, 853-973 step_head_tokens_in_place):

  * the native captures' rows (tests/golden/pinned.json): the updated state
    row and output bit for bit, with decay = beta = 1 (the capture's recipe);
  * random heads over several tokens, shared key heads and a batch: every
    output and state element bit for bit against the oracle's restatement
    (oracle/pinned_oracle.c po_pinned_gdn_prefill);
  * a nonfinite input reports E_NONFINITE and the executor recovers.
"""
import json
import os

import numpy as np
import pytest
import torch

import prism_b200 as pb

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def f32(bits):
    return np.array(bits, np.uint32).view(np.float32)


def b32(x):
    return np.asarray(x, np.float32).reshape(-1).view(np.uint32).tolist()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.fixture(scope="module")
def ex():
    e = pb.ProjectionExecutor(0)
    yield e
    e.close()


def run(ex, state, q, k, v, g, b):
    B, H = state.shape[0], state.shape[1]
    T, KH = q.shape[1], q.shape[2]
    S, Q, K, V, G, Bt = map(dev, (state, q, k, v, g, b))
    O = torch.zeros((B, T, H, 128), device="cuda")
    pb.gdn_prefill_pinned_device(ex, B, T, H, KH, S.data_ptr(), Q.data_ptr(), K.data_ptr(),
                                 V.data_ptr(), G.data_ptr(), Bt.data_ptr(), O.data_ptr())
    torch.cuda.synchronize()
    ex.sync()
    return S.cpu().numpy(), O.cpu().numpy()


def test_native_capture_rows(ex):
    with open(os.path.join(HERE, "golden", "pinned.json")) as f:
        cap = json.load(f)
    for i, r in enumerate(cap["gdn"]["rows"]):
        rng = np.random.default_rng(i)
        state = (rng.standard_normal((1, 1, 128, 128)) * 0.05).astype(np.float32)
        state[0, 0, 0] = f32(r["state"])
        q = f32(r["q"]).reshape(1, 1, 1, 128)
        k = f32(r["k"]).reshape(1, 1, 1, 128)
        v = rng.standard_normal((1, 1, 1, 128)).astype(np.float32)
        v[0, 0, 0, 0] = f32([r["v"]])[0]
        one = np.ones((1, 1, 1), np.float32)
        s, o = run(ex, state, q, k, v, one, one)
        assert b32(s[0, 0, 0]) == r["native_state"]
        assert b32(o[0, 0, 0, 0]) == [r["native_out"]]


@pytest.mark.parametrize("B,T,H,KH", [(1, 1, 16, 16), (2, 37, 4, 2), (1, 64, 16, 4)])
def test_matches_the_oracle_bit_for_bit(ex, oracle, B, T, H, KH):
    rng = np.random.default_rng(100 + T)
    q = rng.standard_normal((B, T, KH, 128)).astype(np.float32)
    k = rng.standard_normal((B, T, KH, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, H, 128)).astype(np.float32)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal((B, T, H))))).astype(np.float32)
    bt = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    s0 = (rng.standard_normal((B, H, 128, 128)) * 0.1).astype(np.float32)
    rc, se, oe = oracle.pinned_gdn_prefill(s0, q, k, v, g, bt)
    assert rc == 0
    s, o = run(ex, s0, q, k, v, g, bt)
    assert np.array_equal(s.view(np.uint32), se.view(np.uint32))
    assert np.array_equal(o.view(np.uint32), oe.view(np.uint32))


def test_nonfinite_is_reported(ex):
    rng = np.random.default_rng(5)
    q = rng.standard_normal((1, 2, 1, 128)).astype(np.float32)
    k = q.copy()
    v = rng.standard_normal((1, 2, 1, 128)).astype(np.float32)
    v[0, 1, 0, 9] = np.inf
    one = np.ones((1, 2, 1), np.float32)
    state = np.zeros((1, 1, 128, 128), np.float32)
    with pytest.raises(pb.PrismB200Error) as err:
        run(ex, state, q, k, v, one, one)
    assert err.value.code == pb.E_NONFINITE
    ex.reset()
    v[0, 1, 0, 9] = 0.5
    s, o = run(ex, state, q, k, v, one, one)
    assert np.isfinite(s).all() and np.isfinite(o).all()


def test_long_sequence_matches_the_oracle(ex, oracle):
    """512 tokens, a ragged head count and shared key heads: the recurrence
    stays bit-identical over a long chain."""
    rng = np.random.default_rng(512)
    B, T, H, KH = 1, 512, 6, 3
    q = rng.standard_normal((B, T, KH, 128)).astype(np.float32)
    k = rng.standard_normal((B, T, KH, 128)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, H, 128)).astype(np.float32)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal((B, T, H))))).astype(np.float32)
    bt = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    s0 = np.zeros((B, H, 128, 128), np.float32)
    rc, se, oe = oracle.pinned_gdn_prefill(s0, q, k, v, g, bt)
    assert rc == 0
    s, o = run(ex, s0, q, k, v, g, bt)
    assert np.array_equal(s.view(np.uint32), se.view(np.uint32))
    assert np.array_equal(o.view(np.uint32), oe.view(np.uint32))


def test_refusals_leave_the_buffers_alone(ex):
    """Geometry the reference's pinned step rejects (no tokens, heads not a
    multiple of the key heads), a width other than 128, a misaligned buffer
    and missing gates are refused on the host before anything is enqueued."""
    B, T, H, KH = 1, 2, 2, 1
    S = torch.ones((B, H, 128, 128), device="cuda")
    Q = torch.zeros((B, T, KH, 128), device="cuda")
    V = torch.zeros((B, T, H, 128), device="cuda")
    G = torch.ones((B, T, H), device="cuda")
    O = torch.full((B, T, H, 128), 7.0, device="cuda")
    p = lambda t: t.data_ptr()
    cases = [
        dict(tokens=0), dict(heads=3, key_heads=2), dict(d=64),
        dict(state=p(S) + 4), dict(decay=0), dict(beta=0),
    ]
    for case in cases:
        args = dict(batch=B, tokens=T, heads=H, key_heads=KH, state=p(S), q=p(Q), k=p(Q),
                    v=p(V), decay=p(G), beta=p(G), out=p(O), d=128)
        args.update(case)
        with pytest.raises(pb.PrismB200Error) as err:
            pb.gdn_prefill_pinned_device(ex, args["batch"], args["tokens"], args["heads"],
                                         args["key_heads"], args["state"], args["q"], args["k"],
                                         args["v"], args["decay"], args["beta"], args["out"],
                                         d=args["d"])
        assert err.value.code in (pb.E_INVALID, pb.E_UNSUPPORTED), case
    torch.cuda.synchronize()
    ex.sync()
    assert bool((S == 1).all()) and bool((O == 7).all())
