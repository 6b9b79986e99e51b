"""Decoder checkpoints on the device (the reference's Decoder::checkpoint /
checkpoint_into / restore, src/lib.rs:305-319, src/graph.rs:5483-5578):

  * restore then the same tokens gives the same logits, KV rows and
    recurrent state, bit for bit, under every KV policy and both step modes;
  * a restore after further steps, after a reset, and of a position-0
    checkpoint (a reset);
  * checkpoint_into reuses storage; device-driven generation resumes from a
    restored state exactly as from the original;
  * a checkpoint of another model is refused and leaves the model usable.
"""
import numpy as np
import pytest

import prism_b200 as pb
import qwen35

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def state(gm, cfg):
    out = []
    for l in range(cfg.layers):
        if cfg.is_full(l):
            out.append(gm.read_state(l, 2).tobytes() + gm.read_state(l, 3).tobytes())
        else:
            out.append(gm.read_state(l, 0).tobytes() + gm.read_state(l, 1).tobytes())
    return out


@pytest.mark.parametrize("policy,mode", [(qwen35.KV_F16, "flow"), (qwen35.KV_Q8_0, "seq"),
                                         (qwen35.KV_Q8_0, "flow"), (pb.KV_RSQ4, "seq")])
def test_restore_replays_bit_for_bit(monkeypatch, policy, mode):
    monkeypatch.setenv("PRISM_B200_STEP", mode)
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=61)
    toks = qwen35.prompt_tokens(cfg, 40, seed=62)
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg, kv_policy=policy)
        gm.load(W)
        l0 = gm.evaluate(toks[0])[0]
        gm.reset()
        gm.ingest_block(np.asarray(toks[:30], np.uint32))
        cp = gm.checkpoint()
        assert cp.position == 30 and cp.bytes > 0
        before = state(gm, cfg)
        first = [gm.evaluate(t)[0] for t in toks[30:36]]
        after = state(gm, cfg)
        gm.restore(cp)
        assert gm.position == 30 and state(gm, cfg) == before
        again = [gm.evaluate(t)[0] for t in toks[30:36]]
        for a, b in zip(first, again):
            assert np.array_equal(bits(a), bits(b))
        assert state(gm, cfg) == after
        # from a reset model too
        gm.reset()
        gm.restore(cp)
        assert np.array_equal(bits(gm.evaluate(toks[30])[0]), bits(first[0]))
        # checkpoint_into reuses the storage; a position-0 checkpoint resets
        gm.checkpoint_into(cp)
        assert cp.position == 31
        gm.reset()
        cp0 = gm.checkpoint()
        assert cp0.position == 0
        gm.restore(cp)
        assert gm.position == 31
        gm.restore(cp0)
        assert gm.position == 0
        assert np.array_equal(bits(gm.evaluate(toks[0])[0]), bits(l0))
        cp.close()
        cp0.close()
        gm.close()


def test_generation_resumes_from_a_restored_state():
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=63)
    prompt = np.asarray(qwen35.prompt_tokens(cfg, 12, seed=64), np.uint32)
    with pb.ProjectionExecutor(0) as ex:
        gm = qwen35.Qwen35Model(ex, cfg)
        gm.load(W)
        gm.ingest_block(prompt[:8])
        cp = gm.checkpoint()
        out1 = gm.generate(prompt[8:], 6)
        gm.restore(cp)
        out2 = gm.generate(prompt[8:], 6)
        assert list(out1) == list(out2)
        cp.close()
        gm.close()


def test_foreign_checkpoint_is_refused():
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=65)
    toks = qwen35.prompt_tokens(cfg, 4, seed=66)
    with pb.ProjectionExecutor(0) as ex:
        a = qwen35.Qwen35Model(ex, cfg)
        a.load(W)
        b = qwen35.Qwen35Model(ex, cfg)
        b.load(W)
        for t in toks:
            a.evaluate(t)
        cp = a.checkpoint()
        with pytest.raises(pb.PrismB200Error) as e:
            b.restore(cp)
        assert e.value.code == pb.E_INVALID
        assert b.position == 0
        lb = b.evaluate(toks[0])[0]   # still usable
        b.reset()
        assert np.array_equal(bits(b.evaluate(toks[0])[0]), bits(lb))
        cp.close()
        a.close()
        b.close()


def test_gguf_model_equals_the_bound_model(tmp_path):
    """A model loaded from a GGUF file (prism_b200_model_load_gguf) decodes
    bit for bit as the same weights bound by name."""
    import os
    from gguf_writer import qwen35_file
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=67)
    path = os.path.join(tmp_path, "m.gguf")
    qwen35_file(path, cfg, W)
    toks = qwen35.prompt_tokens(cfg, 6, seed=68)
    with pb.ProjectionExecutor(0) as ex:
        a = qwen35.Qwen35Model(ex, cfg, kv_policy=qwen35.KV_Q8_0)
        a.load(W)
        b = qwen35.Qwen35Model.from_gguf(ex, path, cfg.context, qwen35.KV_Q8_0)
        for t in toks:
            assert np.array_equal(bits(a.evaluate(t)[0]), bits(b.evaluate(t)[0]))
        a.close()
        b.close()
