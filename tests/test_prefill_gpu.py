"""Batched prompt ingestion (prefill_async, ingest_block) against the decode
path's one-token ingestion steps.

The reference's Decoder::ingest_block contract (src/lib.rs:215-247) is
complete state and position equivalence to sequential ingestion, so every
comparison here is bit for bit: the KV rows, the recurrent and convolution
state of every layer, the position, and then the logits, greedy token and
hidden state of the decode step that follows the prompt.  The sequential
path itself is checked against the CPU oracle by the model tests.
"""
import dataclasses

import numpy as np
import pytest

import prism_b200 as pb
import qwen35

pytestmark = pytest.mark.gpu


def _state(gm, cfg):
    """Raw bytes of every layer's state: {(layer, which): bytes}."""
    import ctypes as c
    out = {}
    row = cfg.kv_heads * max(cfg.head_dim * 2, 16 + cfg.head_dim * 2)
    for l in range(cfg.layers):
        kinds = (2, 3) if cfg.is_full(l) else (0, 1)
        for which in kinds:
            cap = max(gm.position, 1) * row if which >= 2 else \
                cfg.ssm_values * cfg.ssm_state * cfg.ssm_state * 4 + \
                cfg.conv_channels * (cfg.conv_kernel - 1) * 4
            buf = np.zeros(cap, np.uint8)
            n = gm.L.prism_b200_model_read_state(gm.h, l, which, buf.ctypes.data, buf.nbytes)
            assert n >= 0, (l, which, n)
            out[(l, which)] = buf[:n].copy()
    return out


def _run(gm, cfg, segments, batched, next_token):
    """Ingest the prompt segments (one prefill call, or that many one-token
    steps, per segment), then one decode step; the state after the prompt
    and the step's outputs."""
    gm.reset()
    for seg in segments:
        gm.set_prompt(seg)
        if batched:
            gm.prefill_async(len(seg))
        else:
            gm.ingest_async(len(seg))
    pos = gm.position
    st = _state(gm, cfg)
    lg, greedy = gm.evaluate(next_token)
    return pos, st, lg, greedy, gm.read_state(0, 4)


def _check(cfg, kv_policy, lengths, seed):
    W = qwen35.synthetic_weights(cfg, seed=seed)
    toks = qwen35.prompt_tokens(cfg, sum(lengths) + 1, seed=seed + 1)
    segments, at = [], 0
    for n in lengths:
        segments.append(np.asarray(toks[at:at + n], np.uint32))
        at += n
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=kv_policy)
        gm.load(W)
        ref = _run(gm, cfg, segments, False, toks[-1])
        got = _run(gm, cfg, segments, True, toks[-1])
        gm.close()
    assert got[0] == ref[0] == sum(lengths)
    for key in ref[1]:
        assert got[1][key].size == ref[1][key].size, key
        assert np.array_equal(got[1][key], ref[1][key]), "state %s differs" % (key,)
    assert np.array_equal(got[2].view(np.uint32), ref[2].view(np.uint32)), "logits differ"
    assert got[3] == ref[3]
    assert np.array_equal(got[4].view(np.uint32), ref[4].view(np.uint32)), "hidden differs"


@pytest.mark.parametrize("kv_policy", [0, 1])
def test_small_prefill_matches_ingestion(kv_policy):
    # an odd first segment: the second starts on the other convolution
    # history buffer and attends over the first segment's rows
    _check(qwen35.SMALL, kv_policy, [77, 150], seed=61)


def test_prefill_spanning_chunks():
    # 2100 tokens: a 2048-token pass, then 52 more over the first pass's rows
    cfg = dataclasses.replace(qwen35.SMALL, context=2200)
    _check(cfg, 1, [2100, 3], seed=63)


def test_single_token_prefill():
    _check(qwen35.SMALL, 0, [1, 1, 2], seed=65)


@pytest.mark.parametrize("kv_policy", [0, 1])
def test_config1_geometry_prefill(kv_policy):
    # 4 query heads per KV head: 4 tokens per attention CTA
    cfg = dataclasses.replace(qwen35.CONFIG1, layers=8)
    _check(cfg, kv_policy, [45, 20], seed=67)


def test_ingest_block_bounds_and_parity():
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=69)
    toks = np.asarray(qwen35.prompt_tokens(cfg, 257, seed=70), np.uint32)
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg)
        gm.load(W)
        # rejected before any state changes: empty, oversized, bad token
        for bad in (toks[:0], toks[:257], np.array([1, cfg.vocab], np.uint32)):
            with pytest.raises(pb.PrismB200Error):
                gm.ingest_block(bad)
            assert gm.position == 0
        gm.ingest_block(toks[:200])
        assert gm.position == 200
        st = _state(gm, cfg)
        gm.reset()
        gm.set_prompt(toks[:200])
        gm.ingest_async(200)
        ref = _state(gm, cfg)
        for key in ref:
            assert np.array_equal(st[key], ref[key]), key
        gm.close()
