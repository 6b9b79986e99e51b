"""The dataflow decode step (one cooperative kernel per token, tagged
activations) against the per-phase kernel sequence.

Both paths run the same arithmetic in the same order, so they must agree bit
for bit: logits, greedy tokens, hidden state, recurrent and convolution state
and KV records, token by token, from position 0 and after a batched prompt
pass, on both KV policies.  The kernel sequence itself is compared with the
CPU oracle in test_model_gpu.py and test_long_context_gpu.py.
"""
import numpy as np
import pytest

import prism_b200 as pb
import qwen35

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype.itemsize == 4 else np.uint8)


def states(gm, cfg):
    out = []
    for l in range(cfg.layers):
        if cfg.is_full(l):
            out += [gm.read_state(l, 2).view(np.uint8), gm.read_state(l, 3).view(np.uint8)]
        else:
            out += [gm.read_state(l, 0), gm.read_state(l, 1)]
    return out


def run(mode, cfg, W, kv_policy, toks, prompt=None, gen=6, monkeypatch=None):
    monkeypatch.setenv("PRISM_B200_STEP", mode)
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=kv_policy)
        gm.load(W)
        assert gm.step_mode == (2 if mode == "flow" else 0)
        if prompt is not None:
            gm.set_prompt(prompt)
            gm.prefill_async(len(prompt))
            ex.sync()
        steps = []
        for t in toks:
            lg, g = gm.evaluate(int(t))
            steps.append((lg.copy(), g, gm.read_state(0, 4).copy()))
        st = states(gm, cfg)
        gm.reset()
        generated = list(gm.generate(toks[:4], gen))
        gm.close()
    return steps, st, generated


def compare(a, b):
    (sa, sta, ga), (sb, stb, gb) = a, b
    for i, ((la, gi, ha), (lb, gj, hb)) in enumerate(zip(sa, sb)):
        assert np.array_equal(bits(la), bits(lb)), "step %d logits" % i
        assert gi == gj, "step %d greedy" % i
        assert np.array_equal(bits(ha), bits(hb)), "step %d hidden" % i
    for j, (x, y) in enumerate(zip(sta, stb)):
        assert np.array_equal(bits(x), bits(y)), "state %d" % j
    assert ga == gb


@pytest.mark.parametrize("kv_policy", [qwen35.KV_F16, qwen35.KV_Q8_0])
def test_small_flow_matches_kernel_sequence(kv_policy, monkeypatch):
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=5)
    toks = qwen35.prompt_tokens(cfg, 40, seed=6)
    compare(run("flow", cfg, W, kv_policy, toks, monkeypatch=monkeypatch),
            run("seq", cfg, W, kv_policy, toks, monkeypatch=monkeypatch))


def test_config1_flow_matches_kernel_sequence(monkeypatch):
    cfg = qwen35.CONFIG1
    W = qwen35.synthetic_weights(cfg, seed=5)
    toks = qwen35.prompt_tokens(cfg, 12, seed=6)
    compare(run("flow", cfg, W, qwen35.KV_F16, toks, monkeypatch=monkeypatch),
            run("seq", cfg, W, qwen35.KV_F16, toks, monkeypatch=monkeypatch))


@pytest.mark.parametrize("kv_policy", [qwen35.KV_F16, qwen35.KV_Q8_0])
def test_config1_flow_after_prompt(kv_policy, monkeypatch):
    """configs[1] at the benchmark's positions: a 511-token batched prompt
    pass, then decode steps at positions 511-522 (the attention's position
    split at hundreds of cached rows per CTA)."""
    cfg = qwen35.CONFIG1
    W = qwen35.synthetic_weights(cfg, seed=9)
    prompt = qwen35.prompt_tokens(cfg, 511, seed=10)
    toks = qwen35.prompt_tokens(cfg, 12, seed=11)
    compare(run("flow", cfg, W, kv_policy, toks, prompt=prompt, monkeypatch=monkeypatch),
            run("seq", cfg, W, kv_policy, toks, prompt=prompt, monkeypatch=monkeypatch))


def test_flow_decode_async_and_timings(monkeypatch):
    """Device-driven greedy decode (graph replays without the host) gives the
    same tokens as the kernel sequence, and a traced step reports its
    per-phase times."""
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=13)
    prompt = qwen35.prompt_tokens(cfg, 20, seed=14)
    outs = []
    for mode in ("flow", "seq"):
        monkeypatch.setenv("PRISM_B200_STEP", mode)
        with pb.ProjectionExecutor(0) as ex:
            gm = qwen35.Qwen35Model(ex, cfg)
            gm.load(W)
            outs.append(list(gm.generate(prompt, 30)))
            if mode == "flow":
                att, ffn, head, total = gm.step_timings()
                assert total > 0 and head > 0 and np.all(ffn > 0) and np.all(att > 0)
                assert total + 1e-3 >= float(np.sum(att) + np.sum(ffn))
            gm.close()
    assert outs[0] == outs[1]


@pytest.mark.parametrize("kv_policy", [qwen35.KV_F16, qwen35.KV_Q8_0])
def test_flow_at_the_longest_flow_context(kv_policy, monkeypatch):
    """The small geometry at a 2048-token context after a 2000-token prompt:
    each CTA of a head scores about 250 cached rows in eight K chunks and
    sums every position's values in sixteen V chunks, the most the dataflow
    attention takes."""
    import dataclasses
    cfg = dataclasses.replace(qwen35.SMALL, context=2048)
    W = qwen35.synthetic_weights(cfg, seed=17)
    prompt = qwen35.prompt_tokens(cfg, 2000, seed=18)
    toks = qwen35.prompt_tokens(cfg, 8, seed=19)
    compare(run("flow", cfg, W, kv_policy, toks, prompt=prompt, gen=4, monkeypatch=monkeypatch),
            run("seq", cfg, W, kv_policy, toks, prompt=prompt, gen=4, monkeypatch=monkeypatch))
