"""A minimal GGUF (version 3) writer for the tests: metadata of the types the
loader reads and tensors in ggml dimension order.  Test infrastructure only."""
import struct

import numpy as np

# GGUF value types
U32, I32, F32, BOOL, STRING, ARRAY, U64 = 4, 5, 6, 7, 8, 9, 10


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    if t == U32:
        return struct.pack("<I", v)
    if t == I32:
        return struct.pack("<i", v)
    if t == F32:
        return struct.pack("<f", v)
    if t == BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == STRING:
        return _str(v)
    if t == U64:
        return struct.pack("<Q", v)
    raise ValueError(t)


def write(path, metadata, tensors, alignment=32, version=3):
    """metadata: {key: (type, value)}, arrays as (ARRAY, (elem_type, [values]));
    tensors: [(name, ggml_type, dims (ggml order), bytes)]."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, (t, v) in metadata.items():
        out += _str(key) + struct.pack("<I", t)
        if t == ARRAY:
            et, vals = v
            out += struct.pack("<IQ", et, len(vals)) + b"".join(_value(et, x) for x in vals)
        else:
            out += _value(t, v)
    offsets, off = [], 0
    for name, gtype, dims, data in tensors:
        offsets.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    for (name, gtype, dims, data), o in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gtype, o)
    out += b"\0" * ((-len(out)) % alignment)
    for (name, gtype, dims, data), o in zip(tensors, offsets):
        out += bytes(data) + b"\0" * ((-len(data)) % alignment)
    with open(path, "wb") as f:
        f.write(out)


def qwen35_file(path, cfg, weights, extra=None, drop=()):
    """A Qwen35 GGUF from a config and a synthetic weight dict (the reference's
    `qwen35.*` keys; packed weights [rows][blocks] -> dims [cols, rows])."""
    md = {
        "general.architecture": (STRING, "qwen35"),
        "qwen35.embedding_length": (U32, cfg.hidden),
        "qwen35.block_count": (U32, cfg.layers),
        "qwen35.attention.head_count": (U32, cfg.heads),
        "qwen35.attention.head_count_kv": (U32, cfg.kv_heads),
        "qwen35.attention.key_length": (U32, cfg.head_dim),
        "qwen35.attention.value_length": (U32, cfg.head_dim),
        "qwen35.rope.dimension_count": (U32, cfg.rope_dim),
        "qwen35.rope.dimension_sections": (ARRAY, (I32, list(cfg.rope_sections))),
        "qwen35.rope.freq_base": (F32, cfg.rope_base),
        "qwen35.attention.layer_norm_rms_epsilon": (F32, cfg.eps),
        "qwen35.feed_forward_length": (U32, cfg.ffn),
        "qwen35.ssm.state_size": (U32, cfg.ssm_state),
        "qwen35.ssm.group_count": (U32, cfg.ssm_groups),
        "qwen35.ssm.time_step_rank": (U32, cfg.ssm_values),
        "qwen35.ssm.conv_kernel": (U32, cfg.conv_kernel),
        "qwen35.ssm.inner_size": (U32, cfg.ssm_state * cfg.ssm_values),
        "qwen35.full_attention_interval": (U32, cfg.full_interval),
    }
    md.update(extra or {})
    for k in drop:
        md.pop(k, None)
    bb = {35: 66, 10: 84}[cfg.weight_kind]
    tensors = []
    for name, arr in weights.items():
        if arr.dtype == np.uint8:
            rows = arr.shape[0]
            cols = arr.shape[1] // bb * 256
            tensors.append((name, cfg.weight_kind, [cols, rows], arr.tobytes()))
        else:
            a = np.ascontiguousarray(arr, np.float32)
            dims = list(a.shape[::-1])
            tensors.append((name, 0, dims, a.tobytes()))
    write(path, md, tensors)
    return md, tensors
