"""GGUF model files (the reference's Model::load, src/model.rs:266-420, and
the Qwen35 geometry of src/graph.rs:2966-3100), parsed on the host: the
geometry from the `qwen35.*` keys, every tensor's bytes, and the refusals of
malformed or unsupported files."""
import os
import struct

import numpy as np
import pytest

import prism_b200 as pb
import qwen35
from gguf_writer import ARRAY, BOOL, I32, U32, qwen35_file, write


def small(tmp_path, **kw):
    cfg = qwen35.SMALL
    W = qwen35.synthetic_weights(cfg, seed=3)
    path = os.path.join(tmp_path, "m.gguf")
    md, tensors = qwen35_file(path, cfg, W, **kw)
    return cfg, W, path, tensors


def test_geometry_and_tensors_round_trip(tmp_path):
    cfg, W, path, tensors = small(tmp_path)
    g = qwen35.GgufFile(path)
    got = g.config(256, qwen35.KV_Q8_0)
    for f in ("hidden", "layers", "heads", "kv_heads", "head_dim", "rope_dim", "ffn", "vocab",
              "ssm_state", "ssm_groups", "ssm_values", "conv_kernel", "full_interval",
              "weight_kind"):
        assert getattr(got, f) == getattr(cfg, f), f
    assert got.rope_sections == tuple(cfg.rope_sections)
    assert np.float32(got.rope_base) == np.float32(cfg.rope_base)
    assert np.float32(got.eps) == np.float32(cfg.eps)
    assert got.context == 256
    back = g.tensors()
    assert [t[0] for t in back] == [t[0] for t in tensors]
    for (name, typ, dims, data), (n2, t2, d2, b2) in zip(back, tensors):
        assert (typ, dims, data) == (t2, d2, b2), name
    g.close()


def test_recurrent_layer_flags_must_follow_the_interval(tmp_path):
    cfg = qwen35.SMALL
    flags = [(l + 1) % cfg.full_interval != 0 for l in range(cfg.layers)]
    _, _, path, _ = small(tmp_path, extra={"qwen35.attention.recurrent_layers":
                                           (ARRAY, (BOOL, flags))})
    qwen35.GgufFile(path).config(64)
    flags[0] = not flags[0]
    _, _, path, _ = small(tmp_path, extra={"qwen35.attention.recurrent_layers":
                                           (ARRAY, (BOOL, flags))})
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.GgufFile(path).config(64)
    assert e.value.code == pb.E_UNSUPPORTED


@pytest.mark.parametrize("drop", ["qwen35.ssm.inner_size", "qwen35.rope.dimension_sections",
                                  "qwen35.attention.key_length"])
def test_missing_keys_are_refused(tmp_path, drop):
    _, _, path, _ = small(tmp_path, drop=(drop,))
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.GgufFile(path).config(64)
    assert e.value.code == pb.E_INVALID and drop.split(".")[-1] in str(e.value)


def test_malformed_files_are_refused(tmp_path):
    p = os.path.join(tmp_path, "x.gguf")
    cases = {
        "magic": b"GGUX" + struct.pack("<IQQ", 3, 0, 0),
        "version": b"GGUF" + struct.pack("<IQQ", 7, 0, 0),
        "truncated": b"GGUF" + struct.pack("<I", 3),
    }
    for name, blob in cases.items():
        with open(p, "wb") as f:
            f.write(blob)
        with pytest.raises(pb.PrismB200Error):
            qwen35.GgufFile(p)
    # a tensor past the end of the file, an unknown type, a partial block,
    # a duplicate name
    ok = np.zeros(4, np.float32).tobytes()
    for tensors in ([("a", 0, [4], ok), ("b", 0, [1 << 20], ok)],
                    [("a", 99, [4], ok)],
                    [("a", 35, [100, 1], bytes(66))],
                    [("a", 0, [4], ok), ("a", 0, [4], ok)]):
        write(p, {"k": (U32, 1)}, tensors)
        if tensors[-1][2] == [1 << 20]:
            with open(p, "r+b") as f:  # shrink the data so b lies outside
                f.truncate(os.path.getsize(p) - 16)
        with pytest.raises(pb.PrismB200Error):
            qwen35.GgufFile(p)
    write(p, {"k": (I32, -1)}, [("a", 0, [4], ok)])
    qwen35.GgufFile(p)  # a valid file without Qwen35 keys opens ...
    with pytest.raises(pb.PrismB200Error):
        qwen35.GgufFile(p).config(64)  # ... and has no geometry


def test_untied_output_head_is_refused(tmp_path):
    cfg = qwen35.SMALL
    W = dict(qwen35.synthetic_weights(cfg, seed=3))
    W["output.weight"] = W["token_embd.weight"]
    path = os.path.join(tmp_path, "m.gguf")
    qwen35_file(path, cfg, W)
    with pytest.raises(pb.PrismB200Error) as e:
        qwen35.GgufFile(path).config(64)
    assert e.value.code == pb.E_UNSUPPORTED
