"""CPU checks of the Qwen35 / GDN oracle (no GPU)."""
import numpy as np
import pytest

import qwen35


def _gdn_inputs(T, width=128, rows=128, seed=0):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, width)).astype(np.float32)
    k = rng.standard_normal((T, width)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    k /= np.linalg.norm(k, axis=1, keepdims=True)
    v = rng.standard_normal((T, rows)).astype(np.float32)
    g = np.exp(-np.log1p(np.exp(rng.standard_normal(T)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal(T)))).astype(np.float32)
    return q, k, v, g, beta


@pytest.mark.parametrize("chunk", [8, 32, 64])
def test_chunkwise_gdn_matches_sequential_recurrence(oracle, chunk):
    """The chunkwise (WY) form agrees with the exact recurrence within the
    reference's chunkwise tolerance 1e-3 + 1e-3*|ref|
    (reference docs/cpu-tiled-prefill.md:173-189)."""
    q, k, v, g, beta = _gdn_inputs(200)
    s0 = np.random.default_rng(9).standard_normal((128, 128)).astype(np.float32) * 0.1
    se, oe = oracle.gdn_head_prefill(s0, q, k, v, g, beta)
    sc, oc = oracle.gdn_head_prefill(s0, q, k, v, g, beta, chunk=chunk)
    assert np.all(np.abs(oc - oe) <= 1e-3 + 1e-3 * np.abs(oe))
    assert np.all(np.abs(sc - se) <= 1e-3 + 1e-3 * np.abs(se))


def test_gdn_step_matches_numpy_definition(oracle):
    q, k, v, g, beta = _gdn_inputs(1)
    prev = np.random.default_rng(2).standard_normal((128, 128)).astype(np.float32)
    nxt, out = oracle.gdn_head_step(prev, q[0], k[0], v[0], float(g[0]), float(beta[0]))
    s = g[0].astype(np.float64) * prev.astype(np.float64)
    delta = (v[0] - s @ k[0]) * beta[0]
    s = s + np.outer(delta, k[0])
    o = (s @ q[0]) / np.sqrt(128)
    assert np.allclose(nxt, s, rtol=1e-5, atol=1e-5)
    assert np.allclose(out, o, rtol=1e-4, atol=1e-5)


def test_small_model_runs_and_is_deterministic(oracle):
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=3)
    m1 = oracle.Qwen35(cfg, W)
    m2 = oracle.Qwen35(cfg, W)
    toks = qwen35.prompt_tokens(cfg, 6, seed=4)
    for t in toks:
        a = m1.step(t, threads=1)
        b = m2.step(t, threads=4)
        assert np.all(np.isfinite(a))
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert m1.position == 6
    assert m1.keys(3).shape == (6, cfg.kv_heads * cfg.head_dim)
    m1.reset()
    a2 = [m1.step(t) for t in toks][-1]
    assert np.array_equal(a2, a)
    assert oracle.greedy(np.array([1, 3, 3, 2], np.float32)) == 1


@pytest.mark.parametrize("policy", [2, 3, 4])
def test_small_model_with_rotated_kv_records(oracle, policy):
    """The rotated scalar KV policies (2 rsq4, 3 rsq4vf, 4 rsq4k3v) store
    every position as a record that decodes near the binary16 policy's row,
    and the logits stay near the binary16 policy's (the codec is lossy)."""
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=3)
    exact = oracle.Qwen35(cfg, W)
    packed = oracle.Qwen35(cfg, W, kv_policy=policy)
    toks = qwen35.prompt_tokens(cfg, 5, seed=4)
    for t in toks:
        a = exact.step(t, threads=2)
        b = packed.step(t, threads=2)
        assert np.all(np.isfinite(b))
    assert np.max(np.abs(a - b)) < 0.1 * max(1.0, np.max(np.abs(a)))
    kb, vb, _ = oracle.KVQ_POLICIES[("rsq4", "rsq4vf", "rsq4k3v")[policy - 2]]
    layer = next(l for l in range(cfg.layers) if (l + 1) % cfg.full_interval == 0)
    keys = packed.records(layer)
    vals = packed.records(layer, value=True)
    assert keys.shape == (5, cfg.kv_heads, 132)
    assert vals.shape == (5, cfg.kv_heads, oracle.kvq_record_bytes(vb))
    ref_k = exact.keys(layer).view(np.float16).astype(np.float32).reshape(5, cfg.kv_heads, 256)
    dec = oracle.kvq_decode(kb, oracle.KVQ_KEY_SEED, keys.reshape(-1, 132)).reshape(ref_k.shape)
    # the first position saw identical inputs under both policies
    err = np.sum((dec[0] - ref_k[0]) ** 2) / np.sum(ref_k[0] ** 2)
    assert err < 0.04
