"""The reference's rotated scalar KV codec ("rsq", src/kv_quant.rs) and the
attention over its records (src/graph/quantized_kv.rs attend_head) on the
device, through the C ABI, against the oracle -- bit for bit:

  * encode: records of 3- and 4-bit codecs, versions 1 and 2, the policies'
    seeds and the reference's fixture seeds, rows of every scale the
    reference's codec tests use (zero, sparse, constant, 1e-39, 1e30);
  * decode: the reconstruction of those records;
  * attention: every policy, 1 to 5000 positions, GQA groups;
  * a malformed record refused with E_INVALID;
  * the model under each rotated policy (one-token steps, the batched
    prompt pass, generation): KV records byte for byte, logits, and the
    greedy tokens.  Model logits follow the tolerance of test_model_gpu.py
    (|gpu - ref| <= 1e-4 + 1e-4 |ref|); the codec and attention are exact.
"""
import numpy as np
import pytest

import prism_b200 as pb
import qwen35

pytestmark = pytest.mark.gpu
KEY, VALUE = pb.KVQ_KEY_SEED, pb.KVQ_VALUE_SEED
POLICY = {pb.KV_RSQ4: "rsq4", pb.KV_RSQ4VF: "rsq4vf", pb.KV_RSQ4K3V: "rsq4k3v"}


def bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def fixture_rows(seed):
    linear = np.arange(256, dtype=np.float32) - np.float32(127.5)
    base = (linear / np.float32(32.0) + np.sin(linear * np.float32(0.17))).astype(np.float32)
    sparse = np.zeros(256, np.float32)
    sparse[19] = 3.0
    rng = np.random.default_rng(seed)
    rows = [base, sparse, np.ones(256, np.float32), np.zeros(256, np.float32),
            (base * np.float32(1e-39)).astype(np.float32),
            (base * np.float32(1e30)).astype(np.float32)]
    rows += list(rng.standard_normal((58, 256)).astype(np.float16).astype(np.float32))
    rows += list((rng.standard_normal((64, 256)) * rng.uniform(1e-3, 1e3, (64, 1)))
                 .astype(np.float32))
    return np.stack(rows)


@pytest.fixture(scope="module")
def ex():
    with pb.ProjectionExecutor(0) as e:
        yield e


@pytest.mark.parametrize("bits,version", [(4, 1), (3, 1), (4, 2), (3, 2)])
@pytest.mark.parametrize("seed", [KEY, VALUE, 42])
def test_encode_and_decode_match_oracle(ex, bits, version, seed):
    from oracle import oracle
    rows = fixture_rows(seed % 1000)
    got = ex.kvq_encode(bits, seed, rows, version=version)
    want = oracle.kvq_encode(bits, seed, rows, version=version)
    assert np.array_equal(got, want)
    dec = ex.kvq_decode(bits, seed, want)
    assert np.array_equal(bits32(dec), bits32(oracle.kvq_decode(bits, seed, want)))


@pytest.mark.parametrize("policy", [pb.KV_RSQ4, pb.KV_RSQ4VF, pb.KV_RSQ4K3V])
@pytest.mark.parametrize("n,heads,kv_heads", [(1, 4, 2), (7, 4, 4), (37, 16, 4),
                                              (300, 8, 1), (2049, 16, 4), (5000, 4, 2)])
@pytest.mark.parametrize("qscale", [2.0, 0.25])
def test_attention_matches_oracle(ex, policy, n, heads, kv_heads, qscale):
    """qscale 2 spreads the scores so that small exponentials force the
    softmax total's in-order path; 0.25 keeps them in its exact-tree range."""
    from oracle import oracle
    kb, vb, ver = oracle.KVQ_POLICIES[POLICY[policy]]
    rng = np.random.default_rng(n * 31 + heads)
    k = rng.standard_normal((n * kv_heads, 256)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((n * kv_heads, 256)).astype(np.float16).astype(np.float32)
    keys = ex.kvq_encode(kb, KEY, k).reshape(n, kv_heads, -1)
    vals = ex.kvq_encode(vb, VALUE, v, version=ver).reshape(n, kv_heads, -1)
    q = (rng.standard_normal((heads, 256)) * qscale).astype(np.float16).astype(np.float32)
    g = rng.standard_normal((heads, 256)).astype(np.float32)
    got = ex.kvq_attend(policy, q, keys, vals, 1 / 16, g)
    want = oracle.kvq_attend(POLICY[policy], q, keys, vals, heads, kv_heads, 1 / 16, g)
    assert np.array_equal(bits32(got), bits32(want))


def test_malformed_record_is_refused(ex):
    rows = fixture_rows(1)[:4]
    keys = ex.kvq_encode(4, KEY, rows).reshape(4, 1, 132)
    vals = ex.kvq_encode(4, VALUE, rows).reshape(4, 1, 132)
    bad = vals.copy()
    bad[2, 0, :4] = np.frombuffer(np.float32(-1.0).tobytes(), np.uint8)
    q = rows[:1]
    with pytest.raises(pb.PrismB200Error) as e:
        ex.kvq_attend(pb.KV_RSQ4, q, keys, bad, 1 / 16, q)
    assert e.value.code == pb.E_INVALID
    ex.reset()
    zero = keys.copy()
    zero[1, 0, :4] = 0
    zero[1, 0, 4] = 1  # a zero scale with a nonzero code
    with pytest.raises(pb.PrismB200Error) as e:
        ex.kvq_decode(4, KEY, zero[:, 0])
    assert e.value.code == pb.E_INVALID
    ex.reset()
    with pytest.raises(pb.PrismB200Error) as e:  # argument errors leave it open
        ex.kvq_attend(7, q, keys, vals, 1 / 16, q)
    assert e.value.code == pb.E_INVALID
    out = ex.kvq_attend(pb.KV_RSQ4, q, keys, vals, 1 / 16, q)
    assert np.all(np.isfinite(out))


def close(a, b, rtol=1e-4, atol=1e-4):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.all(np.abs(a - b) <= atol + rtol * np.abs(b)), float(np.max(np.abs(a - b)))


@pytest.mark.parametrize("policy", [pb.KV_RSQ4, pb.KV_RSQ4VF, pb.KV_RSQ4K3V])
def test_model_with_rotated_kv_matches_oracle(policy):
    from oracle import oracle
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=41)
    toks = qwen35.prompt_tokens(cfg, 40, seed=42)
    om = oracle.Qwen35(cfg, W, kv_policy=policy)
    ref = [om.step(t, threads=8) for t in toks]
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=policy)
        gm.load(W)
        assert gm.step_mode == 0  # rotated records run the kernel sequence
        for i, t in enumerate(toks[:20]):
            lg, greedy = gm.evaluate(t)
            ok, err = close(lg, ref[i])
            assert ok, "step %d err %g" % (i, err)
        # the rest as one batched prompt pass (one-token steps underneath)
        gm.ingest_block(np.asarray(toks[20:39], np.uint32))
        lg, _ = gm.evaluate(toks[39])
        ok, err = close(lg, ref[39])
        assert ok, "after prefill err %g" % err
        for l in range(cfg.layers):
            if cfg.is_full(l):
                assert np.array_equal(gm.records(l), om.records(l)), l
                assert np.array_equal(gm.records(l, value=True), om.records(l, value=True)), l
        # generation from a fresh start equals stepping the oracle greedily
        gm.reset()
        om.reset()
        prompt = toks[:6]
        out = gm.generate(prompt, 5)
        for t in prompt[:-1]:
            om.step(t, threads=8)
        nxt, want = prompt[-1], []
        for _ in range(5):
            nxt = int(np.argmax(om.step(nxt, threads=8)))
            want.append(nxt)
        assert list(out) == want
        gm.close()


def test_batch_refuses_rotated_policy():
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=5)
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=pb.KV_RSQ4)
        gm.load(W)
        with pytest.raises(pb.PrismB200Error) as e:
            qwen35.Qwen35Batch(gm, 2, 64)
        assert e.value.code == pb.E_UNSUPPORTED
        gm.close()
