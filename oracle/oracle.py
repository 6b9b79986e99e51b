"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
the cpu_baseline / --impl reference legs of bench.py, always as the checker
or the timed CPU baseline -- never as the product path.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

Q8K_DTYPE = np.dtype([("scale", "<f4"), ("values", "i1", (256,)), ("sums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292
Q8_0_DTYPE = np.dtype([("d", "<u2"), ("values", "i1", (32,))])
assert Q8_0_DTYPE.itemsize == 34

_lib = None


def build():
    subprocess.check_call(["make", "-s", "-C", HERE])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _declare(L):
    vp, sz, i32, u32, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32, ctypes.c_float
    sig = {
        "po_half_to_float": (f32, [ctypes.c_uint16]),
        "po_float_to_half": (ctypes.c_uint16, [f32]),
        "po_q8k_quantize": (i32, [vp, sz, i32, vp]),
        "po_q8_0_quantize": (i32, [vp, sz, vp]),
        "po_pq2_values": (None, [vp, vp]),
        "po_ptq1_values": (None, [vp, vp]),
        "po_packed_uses_q8k": (i32, [u32, sz]),
        "po_pq2_dot_q8k": (i32, [vp, sz, vp, i32, vp]),
        "po_packed_dot_q8": (i32, [u32, vp, sz, vp, vp]),
        "po_packed_matvec": (i32, [u32, vp, sz, sz, vp, i32, vp]),
        "po_packed_row": (i32, [u32, vp, sz, sz, vp]),
        "po_tq2_decode": (i32, [vp, sz, vp]),
        "po_tq2_quantize": (i32, [vp, sz, vp]),
        "po_tq2_block_dots": (i32, [vp, vp, sz, vp]),
        "po_tq2_dot": (i32, [vp, vp, sz, vp]),
        "po_q2k_decode": (i32, [vp, sz, vp]),
        "po_q2k_block_dots": (i32, [vp, vp, sz, vp, vp]),
        "po_q2k_dot": (i32, [vp, vp, sz, vp]),
        "po_matvec": (i32, [u32, vp, sz, sz, vp, vp, i32]),
        "po_project_tokens": (i32, [u32, vp, sz, sz, vp, sz, i32, vp, i32]),
        "po_float_dot": (f32, [vp, vp, sz]),
        "po_f16_dot": (f32, [vp, vp, sz]),
        "po_silu": (f32, [f32]),
        "po_sigmoid": (f32, [f32]),
        "po_recurrent_decay": (i32, [f32, f32, f32, vp]),
        "po_rms_norm": (i32, [vp, vp, sz, f32, vp]),
        "po_add_rms_norm": (i32, [vp, vp, vp, sz, f32, vp]),
        "po_l2_norm": (None, [vp, sz, f32]),
        "po_softmax_round_f16": (i32, [vp, sz]),
        "po_ext_block_bytes": (i32, [u32]),
        "po_ext_decode": (i32, [u32, vp, sz, vp]),
        "po_ext_block_ints": (i32, [u32, vp, vp, sz, vp, vp]),
        "po_ext_dot": (i32, [u32, vp, vp, sz, vp]),
        "po_tq_quantize": (i32, [u32, vp, sz, vp]),
        "po_gdn_delta_values": (i32, [vp] * 13),
        "po_gdn_delta_values_outputs": (sz, [vp]),
        "po_kvq_splitmix": (ctypes.c_uint64, [vp]),
        "po_kvq_levels": (None, [i32, vp]),
        "po_kvq_record_bytes": (i32, [i32]),
        "po_kvq_encode": (i32, [i32, ctypes.c_uint64, i32, vp, vp]),
        "po_kvq_rotate": (i32, [i32, ctypes.c_uint64, vp, vp]),
        "po_kvq_inverse": (i32, [i32, ctypes.c_uint64, vp]),
        "po_kvq_score": (i32, [i32, vp, vp, vp]),
        "po_kvq_accumulate": (i32, [i32, vp, f32, vp]),
        "po_kvq_decode": (i32, [i32, ctypes.c_uint64, vp, vp]),
        "po_kvq_attend_head": (i32, [i32, ctypes.c_uint64, i32, ctypes.c_uint64, vp, vp, vp, sz,
                                     f32, vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


class OracleError(RuntimeError):
    pass


def _check(st):
    if st != 0:
        raise OracleError("oracle status %d" % st)


def q8k_quantize(x, pinned=False):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 256, dtype=Q8K_DTYPE)
    _check(lib().po_q8k_quantize(_p(x), x.size, int(pinned), _p(out)))
    return out


def q8_0_quantize(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32, dtype=Q8_0_DTYPE)
    _check(lib().po_q8_0_quantize(_p(x), x.size, _p(out)))
    return out


# Q8_K-contract kinds (reference src/kernels.rs:1653-1674): TQ2_0, Q2_K, and
# TQ1_0, Q3_K, Q4_K, Q5_K, Q6_K (kquant_oracle.c)
BLOCK_BYTES = {35: 66, 10: 84, 34: 54, 11: 110, 12: 144, 13: 176, 14: 210}


def block_bytes(kind):
    return BLOCK_BYTES[kind]


# ---- PQ2 (142) and PTQ1 (143): 128 weights per block --------------------
PACKED_BLOCK_BYTES = {142: 34, 143: 28}


def packed_values(kind, block):
    """The 128 weights (-1..2) of one PQ2 or PTQ1 block."""
    b = np.ascontiguousarray(block, dtype=np.uint8)
    out = np.zeros(128, np.int16)
    (lib().po_pq2_values if kind == 142 else lib().po_ptq1_values)(_p(b), _p(out))
    return out


def packed_uses_q8k(kind, cols):
    """The reference's activation contract: Q8_K for PQ2 with a multiple of
    256 columns, Q8_0 otherwise."""
    return bool(lib().po_packed_uses_q8k(kind, cols))


def pq2_dot_q8k(weights_row, act, fused=False):
    w = np.ascontiguousarray(weights_row, dtype=np.uint8)
    a = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    out = np.zeros(1, np.float32)
    _check(lib().po_pq2_dot_q8k(_p(w), w.size // 34, _p(a), int(fused), _p(out)))
    return out[0]


def packed_dot_q8(kind, weights_row, act):
    w = np.ascontiguousarray(weights_row, dtype=np.uint8)
    a = np.ascontiguousarray(act, dtype=Q8_0_DTYPE)
    out = np.zeros(1, np.float32)
    _check(lib().po_packed_dot_q8(kind, _p(w), w.size // PACKED_BLOCK_BYTES[kind], _p(a), _p(out)))
    return out[0]


def packed_matvec(kind, weights, rows, cols, x, fused=False):
    """y = W x for a PQ2 or PTQ1 tensor [rows][cols], x quantized by the
    activation contract of (kind, cols)."""
    w = np.ascontiguousarray(weights, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, np.float32)
    _check(lib().po_packed_matvec(kind, _p(w), rows, cols, _p(x), int(fused), _p(y)))
    return y


def packed_row(kind, weights, cols, r):
    w = np.ascontiguousarray(weights, dtype=np.uint8)
    out = np.zeros(cols, np.float32)
    _check(lib().po_packed_row(kind, _p(w), cols, r, _p(out)))
    return out


def decode(kind, packed):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    nb = packed.size // block_bytes(kind)
    out = np.zeros(nb * 256, dtype=np.float32)
    if kind in (35, 10):
        fn = lib().po_tq2_decode if kind == 35 else lib().po_q2k_decode
        _check(fn(_p(packed), nb, _p(out)))
    else:
        _check(lib().po_ext_decode(kind, _p(packed), nb, _p(out)))
    return out


def tq2_quantize(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 256 * 66, dtype=np.uint8)
    _check(lib().po_tq2_quantize(_p(x), x.size, _p(out)))
    return out


def tq_quantize(kind, x):
    """f32 -> TQ1_0 (34) or TQ2_0 (35) blocks (reference tquants::quantize)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 256 * {34: 54, 35: 66}[kind], dtype=np.uint8)
    _check(lib().po_tq_quantize(kind, _p(x), x.size, _p(out)))
    return out


def dot(kind, packed_row, act):
    packed_row = np.ascontiguousarray(packed_row, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    out = np.zeros(1, dtype=np.float32)
    if kind in (35, 10):
        fn = lib().po_tq2_dot if kind == 35 else lib().po_q2k_dot
        _check(fn(_p(packed_row), _p(act), act.size, _p(out)))
    else:
        _check(lib().po_ext_dot(kind, _p(packed_row), _p(act), act.size, _p(out)))
    return out[0]


def block_dots(kind, packed_row, act):
    """Exact per-block integer dots.  TQ2_0: one int32 per block.
    Q2_K: (isum, msum) int32 pairs per block."""
    packed_row = np.ascontiguousarray(packed_row, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    if kind == 35:
        out = np.zeros(act.size, dtype=np.int32)
        _check(lib().po_tq2_block_dots(_p(packed_row), _p(act), act.size, _p(out)))
        return out
    isum = np.zeros(act.size, dtype=np.int32)
    msum = np.zeros(act.size, dtype=np.int32)
    _check(lib().po_q2k_block_dots(_p(packed_row), _p(act), act.size, _p(isum), _p(msum)))
    return isum, msum


def ext_block_ints(kind, packed_row, act):
    """Exact integer parts per block (kinds 34, 11-14): 8 lane sums
    (TQ1_0: the block sum in lane 0) and the minimum sum (Q4_K, Q5_K)."""
    packed_row = np.ascontiguousarray(packed_row, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    lanes = np.zeros((act.size, 8), dtype=np.int32)
    msum = np.zeros(act.size, dtype=np.int32)
    _check(lib().po_ext_block_ints(kind, _p(packed_row), _p(act), act.size, _p(lanes),
                                   _p(msum)))
    return lanes, msum


def matvec(kind, weights, rows, cols, act, threads=1):
    weights = np.ascontiguousarray(weights, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    y = np.zeros(rows, dtype=np.float32)
    _check(lib().po_matvec(kind, _p(weights), rows, cols, _p(act), _p(y), threads))
    return y


def project_tokens(kind, weights, rows, cols, x, pinned=False, threads=1):
    """y [tokens][rows]: every token quantized to Q8_K and projected."""
    weights = np.ascontiguousarray(weights, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
    y = np.zeros((x.shape[0], rows), dtype=np.float32)
    _check(lib().po_project_tokens(kind, _p(weights), rows, cols, _p(x), x.shape[0],
                                   int(pinned), _p(y), threads))
    return y


def float_dot(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return lib().po_float_dot(_p(a), _p(b), a.size)


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    _check(lib().po_rms_norm(_p(x), _p(w), x.size, eps, _p(out)))
    return out


def softmax_round_f16(v):
    v = np.array(v, dtype=np.float32)
    _check(lib().po_softmax_round_f16(_p(v), v.size))
    return v


# ---- rotated scalar KV codec (kvq_oracle.c) --------------------------------
KVQ_KEY_SEED = 0x5357_4946_544b_5631
KVQ_VALUE_SEED = 0x5357_4946_5456_5631
# policy -> (key bits, value bits, value version)
KVQ_POLICIES = {"rsq4": (4, 4, 1), "rsq4vf": (4, 4, 2), "rsq4k3v": (4, 3, 1)}


def kvq_levels(bits):
    out = np.zeros(16, np.float32)
    lib().po_kvq_levels(8 if bits == 3 else 16, _p(out))
    return out


def kvq_record_bytes(bits):
    return lib().po_kvq_record_bytes(bits)


def kvq_encode(bits, seed, rows, version=1):
    """Records (n, 100|132) uint8 of rows (n, 256) float32."""
    rows = np.ascontiguousarray(np.atleast_2d(rows), np.float32)
    out = np.zeros((rows.shape[0], kvq_record_bytes(bits)), np.uint8)
    for i in range(rows.shape[0]):
        _check(lib().po_kvq_encode(bits, seed, version, _p(rows[i]), _p(out[i])))
    return out


def kvq_rotate(bits, seed, row):
    row = np.ascontiguousarray(row, np.float32)
    out = np.zeros(256, np.float32)
    _check(lib().po_kvq_rotate(bits, seed, _p(row), _p(out)))
    return out


def kvq_inverse(bits, seed, row):
    out = np.array(row, np.float32, copy=True)
    _check(lib().po_kvq_inverse(bits, seed, _p(out)))
    return out


def kvq_score(bits, rotated_query, record):
    q = np.ascontiguousarray(rotated_query, np.float32)
    r = np.ascontiguousarray(record, np.uint8)
    out = np.zeros(1, np.float32)
    _check(lib().po_kvq_score(bits, _p(q), _p(r), _p(out)))
    return out[0]


def kvq_accumulate(bits, record, weight, out):
    """In-place accumulation of weight * record into out (256 float32)."""
    r = np.ascontiguousarray(record, np.uint8)
    _check(lib().po_kvq_accumulate(bits, _p(r), float(weight), _p(out)))
    return out


def kvq_decode(bits, seed, records):
    records = np.ascontiguousarray(np.atleast_2d(records), np.uint8)
    out = np.zeros((records.shape[0], 256), np.float32)
    for i in range(records.shape[0]):
        _check(lib().po_kvq_decode(bits, seed, _p(records[i]), _p(out[i])))
    return out


def kvq_attend(policy, queries, keys, values, heads, kv_heads, attn_scale, gates):
    """Every query head over n positions of packed K/V records (reference
    src/graph/quantized_kv.rs attend_head): queries (heads, 256), keys
    (n, kv_heads, 132), values (n, kv_heads, 100|132), gates (heads, 256)."""
    kb, vb, _ = KVQ_POLICIES[policy]
    keys = np.ascontiguousarray(keys, np.uint8)
    values = np.ascontiguousarray(values, np.uint8)
    n = keys.shape[0]
    group = heads // kv_heads
    out = np.zeros((heads, 256), np.float32)
    for h in range(heads):
        kh = h // group
        k = np.ascontiguousarray(keys[:, kh])
        v = np.ascontiguousarray(values[:, kh])
        q = np.ascontiguousarray(queries[h], np.float32)
        g = np.ascontiguousarray(gates[h], np.float32)
        _check(lib().po_kvq_attend_head(kb, KVQ_KEY_SEED, vb, KVQ_VALUE_SEED, _p(q), _p(k), _p(v),
                                        n, float(attn_scale), _p(g), _p(out[h])))
    return out


class GdnOp(ctypes.Structure):
    """po_gdn_op: geometry of the batched gated-delta op (gdn_op_oracle.c)."""
    _fields_ = [(n, ctypes.c_uint32) for n in ("width", "heads", "tokens", "sequences",
                                               "q_heads", "k_heads", "q_sequences",
                                               "k_sequences", "gate_width", "snapshots")] + \
               [("raw", ctypes.c_int32), ("replay", ctypes.c_int32),
                ("state_rows", ctypes.c_uint32), ("record_banks", ctypes.c_uint32),
                ("record_bank_elems", ctypes.c_uint64), ("records_len", ctypes.c_uint64)]


def gdn_delta_values(op, q, k, v, gate, beta, table, rows=None, bias=None, weight=None,
                     records=None, control=None):
    """The reference's CpuBackend::delta_values (operation 100, or 101 when
    op.replay): returns the flat output (attention rows, then snapshots or
    the replay state and records)."""
    L = lib()
    f = lambda a: None if a is None else np.ascontiguousarray(a, np.float32)
    i = lambda a: None if a is None else np.ascontiguousarray(a, np.int32)
    arrs = [f(q), f(k), f(v), f(gate), f(beta), f(table), i(rows), f(bias), f(weight),
            f(records), i(control)]
    out = np.zeros(L.po_gdn_delta_values_outputs(ctypes.byref(op)), np.float32)
    ptrs = [None if a is None else _p(a) for a in arrs]
    _check(L.po_gdn_delta_values(ctypes.byref(op), *ptrs, _p(out)))
    return out


def recurrent_decay(alpha, time_bias, decay_weight):
    out = np.zeros(1, dtype=np.float32)
    _check(lib().po_recurrent_decay(alpha, time_bias, decay_weight, _p(out)))
    return out[0]


# ---- Qwen35 model oracle ----------------------------------------------------

class _Cfg(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("layers", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("rope_dim", ctypes.c_int32), ("rope_sections", ctypes.c_int32 * 4),
                ("rope_base", ctypes.c_float), ("eps", ctypes.c_float), ("ffn", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("ssm_state", ctypes.c_int32),
                ("ssm_groups", ctypes.c_int32), ("ssm_values", ctypes.c_int32),
                ("conv_kernel", ctypes.c_int32), ("full_interval", ctypes.c_int32),
                ("context", ctypes.c_int32), ("weight_kind", ctypes.c_uint32),
                ("kv_policy", ctypes.c_uint32)]


W_SLOTS = ["attn_norm.weight", "post_attention_norm.weight", "ffn_gate.weight", "ffn_up.weight",
           "ffn_down.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight",
           "attn_output.weight", "attn_q_norm.weight", "attn_k_norm.weight", "attn_qkv.weight",
           "attn_gate.weight", "ssm_beta.weight", "ssm_alpha.weight", "ssm_out.weight",
           "ssm_conv1d.weight", "ssm_dt.bias", "ssm_a", "ssm_norm.weight"]


def _model_lib():
    L = lib()
    if not getattr(L, "_model_declared", False):
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        for name, res, args in [
            ("po_qwen35_create", vp, [vp, vp, vp]), ("po_qwen35_destroy", None, [vp]),
            ("po_qwen35_reset", None, [vp]), ("po_qwen35_step", i32, [vp, ctypes.c_uint32, vp, i32]),
            ("po_qwen35_position", ctypes.c_int32, [vp]),
            ("po_qwen35_conv_state", vp, [vp, i32]), ("po_qwen35_matrix_state", vp, [vp, i32]),
            ("po_qwen35_keys", vp, [vp, i32]), ("po_qwen35_values", vp, [vp, i32]),
            ("po_qwen35_hidden", vp, [vp]), ("po_greedy", i32, [vp, ctypes.c_size_t, vp]),
            ("po_gdn_head_step", i32, [vp, vp, vp, vp, vp, ctypes.c_float, ctypes.c_float, i32, i32, vp]),
            ("po_gdn_head_prefill_exact", i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, vp]),
            ("po_gdn_head_prefill_chunked", i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
            ("po_rope_frequencies", None, [vp, i32, vp]),
            ("po_qwen35_load_state", i32, [vp, i32, i32, vp, ctypes.c_size_t]),
            ("po_qwen35_set_position", i32, [vp, ctypes.c_int32]),
            ("po_pinned_gdn_dot", ctypes.c_float, [vp, vp, ctypes.c_size_t]),
            ("po_pinned_gdn_add_scaled", i32, [vp, vp, ctypes.c_float, ctypes.c_size_t]),
            ("po_pinned_gdn_prefill", i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
            ("po_pinned_attention_dot", i32, [vp, vp, ctypes.c_size_t, vp]),
            ("po_vector_exp", ctypes.c_float, [ctypes.c_float]),
            ("po_pinned_softmax", i32, [vp, ctypes.c_size_t, i32]),
            ("po_pinned_rope", i32, [vp, ctypes.c_size_t, i32, i32, vp, i32]),
            ("po_source_rope", i32, [vp, ctypes.c_size_t, i32, i32, vp]),
            ("po_synth_weights", i32, [ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint64,
                                       ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float,
                                       ctypes.c_float, vp]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        L._model_declared = True
    return L


def make_cfg(cfg, kv_policy=0):
    c = _Cfg()
    for f, _ in _Cfg._fields_:
        if f == "rope_sections":
            c.rope_sections = (ctypes.c_int32 * 4)(*cfg.rope_sections)
        elif f == "kv_policy":
            c.kv_policy = kv_policy
        else:
            setattr(c, f, getattr(cfg, f))
    return c


class Qwen35:
    """The reference decode step on the CPU (Source arithmetic)."""

    def __init__(self, cfg, weights, kv_policy=0):
        L = _model_lib()
        self.cfg = cfg
        self._keep = {k: np.ascontiguousarray(v) for k, v in weights.items()}
        self._c = make_cfg(cfg, kv_policy)
        g = (ctypes.c_void_p * 2)(self._keep["token_embd.weight"].ctypes.data,
                                  self._keep["output_norm.weight"].ctypes.data)
        n = cfg.layers * len(W_SLOTS)
        arr = (ctypes.c_void_p * n)()
        for l in range(cfg.layers):
            for s, name in enumerate(W_SLOTS):
                a = self._keep.get("blk.%d.%s" % (l, name))
                arr[l * len(W_SLOTS) + s] = a.ctypes.data if a is not None else None
        self._g, self._arr = g, arr
        self.h = L.po_qwen35_create(ctypes.byref(self._c), g, arr)
        self.L = L

    def close(self):
        if self.h:
            self.L.po_qwen35_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def reset(self):
        self.L.po_qwen35_reset(self.h)

    @property
    def position(self):
        return self.L.po_qwen35_position(self.h)

    def step(self, token, logits=True, threads=8):
        out = np.zeros(self.cfg.vocab, np.float32) if logits else None
        st = self.L.po_qwen35_step(self.h, int(token), _p(out) if logits else None, threads)
        _check(st)
        return out

    def load_state(self, position, states):
        """Continue from a state produced elsewhere: `states` maps
        (layer, which) -> array (which: 0 conv, 1 matrix, 2 keys, 3 values,
        the layouts of conv_state / matrix_state / keys / values)."""
        for (layer, which), arr in states.items():
            a = np.ascontiguousarray(arr)
            _check(self.L.po_qwen35_load_state(self.h, layer, which, _p(a), a.nbytes))
        _check(self.L.po_qwen35_set_position(self.h, int(position)))

    def hidden(self):
        p = self.L.po_qwen35_hidden(self.h)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)),
                                     (self.cfg.hidden,)).copy()

    def matrix_state(self, layer):
        c = self.cfg
        p = self.L.po_qwen35_matrix_state(self.h, layer)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)),
                                     (c.ssm_values, c.ssm_state, c.ssm_state)).copy()

    def conv_state(self, layer):
        c = self.cfg
        p = self.L.po_qwen35_conv_state(self.h, layer)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)),
                                     (c.conv_channels, c.conv_kernel - 1)).copy()

    def keys(self, layer):
        c = self.cfg
        p = self.L.po_qwen35_keys(self.h, layer)
        n = self.position
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint16)),
                                     (c.context, c.kv_heads * c.head_dim))[:n].copy()

    def values(self, layer):
        c = self.cfg
        p = self.L.po_qwen35_values(self.h, layer)
        n = self.position
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint16)),
                                     (c.context, c.kv_heads * c.head_dim))[:n].copy()

    def records(self, layer, value=False):
        """Rotated scalar KV records (kv_policy 2-4) of the cached positions:
        uint8 (position, kv_heads, record bytes)."""
        c = self.cfg
        kb, vb, _ = KVQ_POLICIES[("rsq4", "rsq4vf", "rsq4k3v")[self._c.kv_policy - 2]]
        rb = kvq_record_bytes(vb if value else kb)
        p = (self.L.po_qwen35_values if value else self.L.po_qwen35_keys)(self.h, layer)
        n = self.position
        raw = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint8)),
                                    (c.context * c.kv_heads * c.head_dim * 2,))
        return raw[:n * c.kv_heads * rb].reshape(n, c.kv_heads, rb).copy()


def synth_weights(kind, rows, cols, seed, stream=0, scale_lo=0.01, scale_hi=0.05):
    """Seeded synthetic packed weights on the host (the product library's
    generator restated): uint8 (rows, cols/256*block) in the reference byte
    layout."""
    out = np.empty((rows, cols // 256 * block_bytes(kind)), np.uint8)
    _check(_model_lib().po_synth_weights(kind, rows, cols, seed, stream, scale_lo, scale_hi,
                                         _p(out)))
    return out


# ---- pinned (Swift) variants, for the reference's native captures ----------

def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def pinned_gdn_dot(a, b):
    a, b = _f32(a), _f32(b)
    return np.float32(_model_lib().po_pinned_gdn_dot(_p(a), _p(b), a.size))


def pinned_gdn_add_scaled(target, inp, scale):
    t, x = _f32(target).copy(), _f32(inp)
    _check(_model_lib().po_pinned_gdn_add_scaled(_p(t), _p(x), float(scale), t.size))
    return t


def pinned_gdn_prefill(state, q, k, v, decay, beta):
    """The pinned (Swift) GDN recurrence over every head and token in the
    device layout: state [B][H][d][d], q, k [B][T][KH][d], v [B][T][H][d],
    decay, beta [B][T][H]; returns (status, new state, out [B][T][H][d])."""
    st = np.array(state, np.float32, copy=True)
    B, H, d = st.shape[0], st.shape[1], st.shape[2]
    T, KH = q.shape[1], q.shape[2]
    out = np.zeros((B, T, H, d), np.float32)
    arrs = [np.ascontiguousarray(x, np.float32) for x in (q, k, v, decay, beta)]
    rc = _model_lib().po_pinned_gdn_prefill(_p(st), *[_p(x) for x in arrs], B, T, H, KH, d,
                                            _p(out))
    return rc, st, out


def pinned_attention_dot(values, weights):
    v, w = _f32(values), _f32(weights)
    out = np.zeros(1, np.float32)
    _check(_model_lib().po_pinned_attention_dot(_p(v), _p(w), w.size, _p(out)))
    return out[0]


def vector_exp(x):
    return np.float32(_model_lib().po_vector_exp(float(np.float32(x))))


def pinned_softmax(scores, round_f16=False):
    s = _f32(scores).copy()
    _check(_model_lib().po_pinned_softmax(_p(s), s.size, int(round_f16)))
    return s


def pinned_rope(x, cos_sin, head=256, rotary=64, in_place=False):
    v, cs = _f32(x).copy(), _f32(cos_sin)
    _check(_model_lib().po_pinned_rope(_p(v), v.size, head, rotary, _p(cs), int(in_place)))
    return v


def source_rope(x, cos_sin, head=256, rotary=64):
    v, cs = _f32(x).copy(), _f32(cos_sin)
    _check(_model_lib().po_source_rope(_p(v), v.size, head, rotary, _p(cs)))
    return v


def greedy(logits):
    out = np.zeros(1, np.uint32)
    _check(_model_lib().po_greedy(_p(np.ascontiguousarray(logits, np.float32)), logits.size, _p(out)))
    return int(out[0])


def gdn_head_step(prev, q, k, v, decay, beta):
    rows, width = prev.shape
    nxt = np.zeros_like(prev)
    out = np.zeros(rows, np.float32)
    _check(_model_lib().po_gdn_head_step(_p(prev), _p(nxt), _p(q), _p(k), _p(v), decay, beta,
                                         rows, width, _p(out)))
    return nxt, out


def gdn_head_prefill(state, q, k, v, decay, beta, chunk=None):
    """q, k: [T][width]; v: [T][rows]; returns (new state, out [T][rows])."""
    state = np.array(state, np.float32, copy=True)
    T, width = q.shape
    rows = v.shape[1]
    out = np.zeros((T, rows), np.float32)
    args = [_p(state), _p(np.ascontiguousarray(q, np.float32)), _p(np.ascontiguousarray(k, np.float32)),
            _p(np.ascontiguousarray(v, np.float32)), _p(np.ascontiguousarray(decay, np.float32)),
            _p(np.ascontiguousarray(beta, np.float32)), T, rows, width]
    if chunk is None:
        _check(_model_lib().po_gdn_head_prefill_exact(*args, _p(out)))
    else:
        _check(_model_lib().po_gdn_head_prefill_chunked(*args, chunk, _p(out)))
    return state, out
