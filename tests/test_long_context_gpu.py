"""Long-context parity against the CPU oracle.

The split-context paths only show at long context: the decode attention's
8-CTA position split and its combine, the batched prefill's value pass cut at
the split's rank boundaries, 2048-token prefill passes that a prompt spans,
and the serving attention's per-(sequence, KV head) clusters.  These tests
run each of them at the lengths the benchmark configurations use and compare
with the oracle decoding the same tokens one at a time:

  * the small geometry after a 2100-token prompt (two prefill passes), then
    decode steps at positions 2100-2103, both KV policies;
  * the configs[1] geometry after its 512-token prompt, then decode steps at
    positions 512-517 (the benchmark's positions);
  * batched serving of two sequences to a 4150-token context.

Bounds are the model tests': |gpu - ref| <= 1e-4 + 1e-4 |ref| for logits,
hidden and recurrent state (observed differences are zero); KV records
exactly; greedy tokens wherever the oracle's top-2 logit gap exceeds 1e-2.
"""
import dataclasses

import numpy as np
import pytest

import prism_b200 as pb
import qwen35

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-4


def close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    err = float(np.max(np.abs(a - b))) if a.size else 0.0
    return bool(np.all(np.abs(a - b) <= ATOL + RTOL * np.abs(b))), err


def check_state(gm, om, cfg, position, kv_policy):
    """KV records of every attention layer and recurrent / convolution state
    of every GDN layer, after `position` tokens."""
    for l in range(cfg.layers):
        if cfg.is_full(l):
            for which, ref in ((2, om.keys(l)), (3, om.values(l))):
                got = gm.read_state(l, which).view(np.uint8).reshape(-1)
                want = np.ascontiguousarray(ref).view(np.uint8).reshape(-1)
                n = position * cfg.kv_heads * (
                    cfg.head_dim // 32 * 2 + cfg.head_dim if kv_policy else 2 * cfg.head_dim)
                assert np.array_equal(got[:n], want[:n]), (l, which)
        else:
            ok, err = close(gm.read_state(l, 1), om.matrix_state(l))
            assert ok, "layer %d recurrent state err %g" % (l, err)
            ok, err = close(gm.read_state(l, 0), om.conv_state(l))
            assert ok, "layer %d conv state err %g" % (l, err)


def run_prompt_then_decode(cfg, kv_policy, prompt_len, decode, seed, threads):
    from oracle import oracle
    W = qwen35.synthetic_weights(cfg, seed=seed)
    prompt = qwen35.prompt_tokens(cfg, prompt_len, seed=seed + 1)
    cont = qwen35.prompt_tokens(cfg, decode, seed=seed + 2)
    om = oracle.Qwen35(cfg, W, kv_policy=kv_policy)
    for t in prompt:
        om.step(int(t), logits=False, threads=threads)
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=kv_policy)
        gm.load(W)
        gm.set_prompt(prompt)
        gm.prefill_async(prompt_len)
        ex.sync()
        assert gm.position == prompt_len
        # the batched pass's contract is the state (and the next step's
        # outputs), not a hidden vector of the last prompt token
        check_state(gm, om, cfg, prompt_len, kv_policy)
        for i, t in enumerate(cont):
            lg, greedy = gm.evaluate(int(t))
            lr = om.step(int(t), threads=threads)
            ok, err = close(lg, lr)
            assert ok, "position %d logits err %g" % (prompt_len + i, err)
            top = np.sort(lr)[-2:]
            if top[1] - top[0] > 1e-2:
                assert greedy == int(np.argmax(lr)), "position %d greedy" % (prompt_len + i)
            ok, err = close(gm.read_state(0, 4), om.hidden())
            assert ok, "position %d hidden err %g" % (prompt_len + i, err)
        check_state(gm, om, cfg, prompt_len + decode, kv_policy)
        gm.close()
    om.close()


@pytest.mark.parametrize("kv_policy", [qwen35.KV_F16, qwen35.KV_Q8_0])
def test_small_after_2100_token_prompt(kv_policy):
    cfg = dataclasses.replace(qwen35.SMALL, context=2304)
    run_prompt_then_decode(cfg, kv_policy, prompt_len=2100, decode=4, seed=61, threads=8)


def test_config1_at_benchmark_positions():
    """the 512-token prompt as one batched pass, then decode at
    positions 512-517, where the benchmark times its steps."""
    run_prompt_then_decode(qwen35.CONFIG1, qwen35.KV_F16, prompt_len=512, decode=6, seed=71,
                           threads=16)


@pytest.mark.parametrize("kv_policy", [qwen35.KV_Q8_0, qwen35.KV_F16])
def test_serving_attention_at_4150_tokens(kv_policy):
    """Two sequences stepped together to a 4150-token context (the serving
    attention's clusters over ~520 positions per CTA); each must match the
    oracle decoding it alone."""
    from oracle import oracle
    cfg = dataclasses.replace(qwen35.SMALL, context=4224)
    steps, B = 4150, 2
    W = qwen35.synthetic_weights(cfg, seed=81)
    toks = [qwen35.prompt_tokens(cfg, steps, seed=82 + i) for i in range(B)]
    oms = [oracle.Qwen35(cfg, W, kv_policy=kv_policy) for _ in range(B)]
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=kv_policy)
        gm.load(W)
        bt = qwen35.Qwen35Batch(gm, B, cfg.context)
        for s in range(steps):
            tail = s >= steps - 3
            greedy = bt.step(np.array([t[s] for t in toks], np.uint32))
            for i in range(B):
                lr = oms[i].step(int(toks[i][s]), logits=tail, threads=8)
                if tail:
                    top = np.sort(lr)[-2:]
                    if top[1] - top[0] > 1e-2:
                        assert greedy[i] == int(np.argmax(lr)), (s, i)
                    ok, err = close(bt.read_state(i, 0, 4), oms[i].hidden())
                    assert ok, "step %d sequence %d hidden err %g" % (s, i, err)
        for i in range(B):
            for l in range(cfg.layers):
                if cfg.is_full(l):
                    for which, ref in ((2, oms[i].keys(l)), (3, oms[i].values(l))):
                        got = bt.read_state(i, l, which)
                        want = np.ascontiguousarray(ref).view(np.uint8).reshape(-1)
                        n = min(got.size, want.size)
                        assert n > 0 and np.array_equal(got[:n], want[:n]), (i, l, which)
                else:
                    ok, err = close(bt.read_state(i, l, 1),
                                    oms[i].matrix_state(l).reshape(-1))
                    assert ok, "sequence %d layer %d state err %g" % (i, l, err)
        bt.close()
        gm.close()
    for om in oms:
        om.close()
