"""Python binding of libprism_b200.so (the C ABI in include/prism_b200.h).

This mirrors the reference's projection-executor seam,
``trait Pq2ProjectionExecutor`` (reference src/kernels/projection.rs:16-350),
for Python callers and for this repository's tests and benchmark: the same
method names (``identity``, ``supports``, ``operation_count``, ``project``,
``project_f32``, ``project_f32_group``), the same argument meaning, and the
same failure behaviour (an error clears the output and closes the executor;
no CPU replay).  All arithmetic runs in the CUDA library; importing this
module on a machine without the built library fails loudly.
"""
import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libprism_b200.so")

OK = 0
E_INVALID, E_UNSUPPORTED, E_NONFINITE, E_DEVICE, E_TIMEOUT, E_FAULTED = 1, 2, 3, 4, 5, 6
KIND_Q2_K, KIND_Q8_K, KIND_TQ2_0 = 10, 15, 35
KIND_PQ2, KIND_PTQ1 = 142, 143   # the reference's own packed ternary formats
BLOCK_BYTES = {KIND_TQ2_0: 66, KIND_Q2_K: 84}
# the rest of the reference's Q8_K contract, served as uploaded (kquant.cuh)
KIND_TQ1_0, KIND_Q3_K, KIND_Q4_K, KIND_Q5_K, KIND_Q6_K = 34, 11, 12, 13, 14
KQUANT_BLOCK_BYTES = {34: 54, 11: 110, 12: 144, 13: 176, 14: 210}   # per 256 weights
PACKED_BLOCK_BYTES = {KIND_PQ2: 34, KIND_PTQ1: 28}   # per 128 weights

Q8K_DTYPE = np.dtype([("scale", "<f4"), ("values", "i1", (256,)), ("sums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292
# prism_b200_q8_block: the reference's Q8Block (scale, code sum, 32 codes)
Q8_DTYPE = np.dtype([("scale", "<f4"), ("sum", "<f4"), ("values", "i1", (32,))])
assert Q8_DTYPE.itemsize == 40


class PrismB200Error(RuntimeError):
    def __init__(self, code, message):
        super().__init__("prism_b200 error %d: %s" % (code, message))
        self.code = code


class _Tensor(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("cols", ctypes.c_uint64),
                ("rows", ctypes.c_uint64), ("data", ctypes.c_void_p)]


_lib = None

# KV policies (include/prism_b200.h): the reference's rotated scalar records
KV_RSQ4, KV_RSQ4VF, KV_RSQ4K3V = 2, 3, 4
KVQ_KEY_SEED = 0x5357_4946_544b_5631
KVQ_VALUE_SEED = 0x5357_4946_5456_5631


def kvq_record_bytes(bits):
    """Record bytes of a codec precision: 100 (3 bits), 132 (4 bits), else 0."""
    return {3: 100, 4: 132}.get(int(bits), 0)


def load():
    """Load the built library; raise if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError("libprism_b200.so is not built: run prism-inference_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    vp, sz, i32, u32, u64, i64 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                  ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64)
    P = ctypes.POINTER
    sig = {
        "prism_b200_executor_create": (i32, [i32, P(vp)]),
        "prism_b200_executor_destroy": (None, [vp]),
        "prism_b200_executor_identity": (ctypes.c_char_p, [vp]),
        "prism_b200_executor_last_error": (sz, [vp, ctypes.c_char_p, sz]),
        "prism_b200_executor_sync": (i32, [vp]),
        "prism_b200_executor_stream": (vp, [vp]),
        "prism_b200_executor_reset": (i32, [vp]),
        "prism_b200_executor_supports": (i32, [vp, P(_Tensor)]),
        "prism_b200_executor_operation_count": (i64, [vp, P(_Tensor)]),
        "prism_b200_weight_upload": (i32, [vp, P(_Tensor), P(vp)]),
        "prism_b200_weight_release": (None, [vp]),
        "prism_b200_project": (i32, [vp, vp, vp, i32, vp]),
        "prism_b200_project_device": (i32, [vp, vp, vp, i32, vp, vp]),
        "prism_b200_project_f32": (i32, [vp, vp, vp, i32, vp]),
        "prism_b200_project_f32_group": (i32, [vp, sz, P(vp), vp, i32, P(vp)]),
        "prism_b200_project_f32_tokens": (i32, [vp, vp, sz, vp, i32, vp]),
        "prism_b200_project_f32_tokens_device": (i32, [vp, vp, sz, vp, i32, vp, vp]),
        "prism_b200_quantize_q8k": (i32, [vp, vp, sz, i32, vp]),
        "prism_b200_quantize_q8k_device": (i32, [vp, vp, sz, i32, vp, vp]),
        "prism_b200_block_dots": (i32, [vp, vp, vp, vp, vp]),
        "prism_b200_synth_weights": (i32, [u32, u64, u64, u64, u64, ctypes.c_float,
                                           ctypes.c_float, vp]),
        "prism_b200_weight_kind": (u32, [vp]),
        "prism_b200_weight_rows": (u64, [vp]),
        "prism_b200_weight_cols": (u64, [vp]),
        "prism_b200_weight_device_bytes": (u64, [vp]),
        "prism_b200_ffn_create": (i32, [vp, vp, vp, vp, u32, u32, u32, P(vp)]),
        "prism_b200_ffn_destroy": (None, [vp]),
        "prism_b200_ffn_exchange_handle": (i32, [vp, vp]),
        "prism_b200_ffn_connect": (i32, [vp, vp]),
        "prism_b200_ffn_chain_tokens": (i32, [vp, sz, vp, vp, i32, vp]),
        "prism_b200_ffn_chain_tokens_device": (i32, [vp, sz, vp, vp, i32, vp, vp]),
        "prism_b200_executor_operation_capacity": (i64, [vp]),
        "prism_b200_tensor_peak_i8": (i32, [vp, i32, P(ctypes.c_double)]),
        "prism_b200_quantize_tq": (i32, [vp, u32, vp, sz, vp]),
        "prism_b200_quantize_tq_device": (i32, [vp, u32, vp, sz, vp, vp]),
        "prism_b200_kvq_record_bytes": (i32, [u32]),
        "prism_b200_kvq_encode": (i32, [vp, u32, u64, u32, vp, sz, vp]),
        "prism_b200_kvq_encode_device": (i32, [vp, u32, u64, u32, vp, sz, vp, vp]),
        "prism_b200_kvq_decode": (i32, [vp, u32, u64, vp, sz, vp]),
        "prism_b200_kvq_attend": (i32, [vp, u32, vp, vp, vp, sz, u32, u32, ctypes.c_float, vp,
                                        vp]),
        "prism_b200_kvq_attend_device": (i32, [vp, u32, vp, vp, vp, sz, u32, u32,
                                               ctypes.c_float, vp, vp, vp]),
        "prism_b200_executor_supports_f32": (i32, [vp, P(_Tensor)]),
        "prism_b200_executor_supports_f32_group": (i32, [vp, sz, P(P(_Tensor))]),
        "prism_b200_executor_supports_q8": (i32, [vp, P(_Tensor)]),
        "prism_b200_project_q8": (i32, [vp, vp, vp, i32, vp]),
        "prism_b200_executor_supports_tile_tokens": (i32, [vp]),
        "prism_b200_project_f32_pair_tokens": (i32, [vp, P(vp), sz, vp, i32, vp, vp]),
        "prism_b200_project_f32_triple_tokens": (i32, [vp, P(vp), sz, vp, i32, vp, vp, vp]),
        "prism_b200_executor_supports_f32_ffn_swiglu": (i32, [vp, P(_Tensor), P(_Tensor)]),
        "prism_b200_project_f32_ffn_swiglu": (i32, [vp, vp, vp, vp, i32, vp]),
        "prism_b200_project_f32_ffn_swiglu_tokens": (i32, [vp, vp, vp, sz, vp, i32, vp]),
        "prism_b200_executor_supports_f32_ffn_chain": (i32, [vp, P(_Tensor), P(_Tensor),
                                                             P(_Tensor)]),
        "prism_b200_project_f32_ffn_chain": (i32, [vp, vp, vp, vp, vp, vp, u32, i32, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def exported_symbols():
    """Names of every function declared in include/prism_b200.h."""
    import re
    hdr = os.path.join(os.path.dirname(HERE), "include", "prism_b200.h")
    with open(hdr) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(prism_b200_\w+)\s*\(", text)))


def synth_weights(kind, rows, cols, seed, stream=0, scale_lo=0.01, scale_hi=0.05):
    """Seeded synthetic packed weights (reference byte layout), generated on
    the host by the library: uint8 array (rows, cols/256*block_bytes)."""
    bb = BLOCK_BYTES[kind]
    out = np.empty((rows, cols // 256 * bb), dtype=np.uint8)
    st = load().prism_b200_synth_weights(kind, rows, cols, seed, stream, scale_lo, scale_hi,
                                         out.ctypes.data)
    if st != OK:
        raise PrismB200Error(st, "invalid synthetic weight request")
    return out


@dataclass
class Tensor:
    """A packed weight in the reference's byte layout (reference
    src/model.rs:184-196): ``cols`` = dimensions[0] (K), ``rows`` = N."""
    kind: int
    cols: int
    rows: int
    data: np.ndarray
    name: str = ""

    def _c(self):
        self.data = np.ascontiguousarray(self.data, dtype=np.uint8)
        return _Tensor(self.kind, self.cols, self.rows, self.data.ctypes.data)


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


class Weight:
    def __init__(self, executor, handle, tensor):
        self.executor = executor
        self.handle = handle
        self.kind, self.cols, self.rows = tensor.kind, tensor.cols, tensor.rows
        self.name = tensor.name

    @property
    def device_bytes(self):
        return load().prism_b200_weight_device_bytes(self.handle)

    def release(self):
        if self.handle:
            load().prism_b200_weight_release(self.handle)
            self.handle = None


class ProjectionExecutor:
    """B200 projection executor (one CUDA device, one stream)."""

    def __init__(self, device=0):
        L = load()
        h = ctypes.c_void_p()
        st = L.prism_b200_executor_create(device, ctypes.byref(h))
        if st != OK:
            raise PrismB200Error(st, "executor create failed on device %d" % device)
        self.h = h
        self._weights = {}

    # -- lifetime --------------------------------------------------------
    def close(self):
        if self.h:
            load().prism_b200_executor_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def last_error(self):
        buf = ctypes.create_string_buffer(1024)
        load().prism_b200_executor_last_error(self.h, buf, 1024)
        return buf.value.decode()

    def _check(self, st):
        if st != OK:
            raise PrismB200Error(st, self.last_error())

    def identity(self):
        return load().prism_b200_executor_identity(self.h).decode()

    def sync(self):
        self._check(load().prism_b200_executor_sync(self.h))

    def stream(self):
        """The executor's cudaStream_t as an integer handle."""
        return load().prism_b200_executor_stream(self.h)

    def reset(self):
        self._check(load().prism_b200_executor_reset(self.h))

    # -- eligibility -----------------------------------------------------
    def supports(self, tensor):
        t = tensor._c()
        return bool(load().prism_b200_executor_supports(self.h, ctypes.byref(t)))

    def operation_count(self, tensor):
        t = tensor._c()
        n = load().prism_b200_executor_operation_count(self.h, ctypes.byref(t))
        return None if n < 0 else n

    def tensor_peak_i8(self, iters=8192):
        """Measured dense int8 tensor-core rate of this device, Tint-op/s
        (no reference counterpart: the GEMM roofline's denominator)."""
        v = ctypes.c_double(0.0)
        self._check(load().prism_b200_tensor_peak_i8(self.h, iters, ctypes.byref(v)))
        return v.value

    def quantize_tq(self, kind, x):
        """f32 weights -> TQ1_0 (34) or TQ2_0 (35) blocks (reference
        src/kernels/tquants.rs:288-336 quantize)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.zeros(x.size // 256 * {34: 54, 35: 66}.get(kind, 1), np.uint8)
        self._check(load().prism_b200_quantize_tq(self.h, kind, _p(x), x.size, _p(out)))
        return out

    # -- rotated scalar KV codec (reference src/kv_quant.rs) --------------
    def kvq_encode(self, bits, seed, rows, version=1):
        """Quantizer::encode of rows (n, 256) float32 -> records (n, 100|132)."""
        rows = np.ascontiguousarray(np.atleast_2d(rows), dtype=np.float32)
        if rows.ndim != 2 or rows.shape[1] != 256:
            raise PrismB200Error(E_INVALID, "codec rows must be [n][256]")
        out = np.zeros((rows.shape[0], max(kvq_record_bytes(bits), 1)), np.uint8)
        self._check(load().prism_b200_kvq_encode(self.h, bits, seed, version, _p(rows),
                                                 rows.shape[0], _p(out)))
        return out

    def kvq_encode_device(self, bits, seed, rows_ptr, n, records_ptr, version=1, stream=None):
        self._check(load().prism_b200_kvq_encode_device(self.h, bits, seed, version, rows_ptr, n,
                                                        records_ptr, stream))

    def kvq_decode(self, bits, seed, records):
        """Quantizer::decode of records (n, 100|132) -> rows (n, 256)."""
        records = np.ascontiguousarray(np.atleast_2d(records), dtype=np.uint8)
        if records.shape[1] != kvq_record_bytes(bits):
            raise PrismB200Error(E_INVALID, "records must be [n][record bytes]")
        out = np.zeros((records.shape[0], 256), np.float32)
        self._check(load().prism_b200_kvq_decode(self.h, bits, seed, _p(records),
                                                 records.shape[0], _p(out)))
        return out

    def kvq_attend(self, policy, queries, keys, values, attn_scale, gates):
        """Gated attention of every query head over packed K/V records
        (reference src/graph/quantized_kv.rs attend_head): queries, gates
        (heads, 256) float32; keys (n, kv_heads, 132), values
        (n, kv_heads, 132|100) uint8."""
        queries = np.ascontiguousarray(queries, dtype=np.float32)
        gates = np.ascontiguousarray(gates, dtype=np.float32)
        keys = np.ascontiguousarray(keys, dtype=np.uint8)
        values = np.ascontiguousarray(values, dtype=np.uint8)
        heads, kv_heads = queries.shape[0], keys.shape[1]
        vbits = 3 if policy == KV_RSQ4K3V else 4
        if (queries.shape != (heads, 256) or gates.shape != queries.shape or keys.ndim != 3
                or keys.shape[2] != 132 or values.shape != keys.shape[:2] +
                (kvq_record_bytes(vbits),)):
            raise PrismB200Error(E_INVALID, "attention extents")
        out = np.zeros((heads, 256), np.float32)
        self._check(load().prism_b200_kvq_attend(self.h, policy, _p(queries), _p(keys),
                                                 _p(values), keys.shape[0], heads, kv_heads,
                                                 float(attn_scale), _p(gates), _p(out)))
        return out

    def kvq_attend_device(self, policy, queries_ptr, keys_ptr, values_ptr, positions, heads,
                          kv_heads, attn_scale, gates_ptr, out_ptr, stream=None):
        self._check(load().prism_b200_kvq_attend_device(
            self.h, policy, queries_ptr, keys_ptr, values_ptr, positions, heads, kv_heads,
            float(attn_scale), gates_ptr, out_ptr, stream))

    def operation_capacity(self):
        """Remaining submissions of a bounded session, None when opaque
        (reference src/kernels/projection.rs:20-28)."""
        n = load().prism_b200_executor_operation_capacity(self.h)
        return None if n < 0 else n

    def supports_f32(self, tensor):
        t = tensor._c()
        return bool(load().prism_b200_executor_supports_f32(self.h, ctypes.byref(t)))

    def supports_f32_group(self, tensors):
        cs = [t._c() for t in tensors]
        arr = (ctypes.POINTER(_Tensor) * len(cs))(*[ctypes.pointer(c) for c in cs])
        return bool(load().prism_b200_executor_supports_f32_group(self.h, len(cs), arr))

    def supports_q8(self, tensor):
        t = tensor._c()
        return bool(load().prism_b200_executor_supports_q8(self.h, ctypes.byref(t)))

    def supports_tile_tokens(self):
        return bool(load().prism_b200_executor_supports_tile_tokens(self.h))

    def supports_f32_ffn_swiglu(self, gate, up):
        g, u = gate._c(), up._c()
        return bool(load().prism_b200_executor_supports_f32_ffn_swiglu(
            self.h, ctypes.byref(g), ctypes.byref(u)))

    def supports_f32_ffn_chain(self, gate, up, down):
        g, u, d = gate._c(), up._c(), down._c()
        return bool(load().prism_b200_executor_supports_f32_ffn_chain(
            self.h, ctypes.byref(g), ctypes.byref(u), ctypes.byref(d)))

    # -- weights ---------------------------------------------------------
    def upload(self, tensor):
        t = tensor._c()
        h = ctypes.c_void_p()
        self._check(load().prism_b200_weight_upload(self.h, ctypes.byref(t), ctypes.byref(h)))
        return Weight(self, h, tensor)

    def _weight(self, w):
        if isinstance(w, Weight):
            return w
        key = id(w)
        if key not in self._weights:
            self._weights[key] = (w, self.upload(w))
        return self._weights[key][1]

    # -- projections -----------------------------------------------------
    def project(self, weight, activation, fused=False):
        """y = W x for prepared Q8_K activation blocks (reference
        src/kernels/projection.rs:48-60)."""
        w = self._weight(weight)
        act = np.ascontiguousarray(activation, dtype=Q8K_DTYPE)
        if act.size * 256 != w.cols:
            raise PrismB200Error(E_INVALID, "activation extent differs from weight columns")
        out = np.zeros(w.rows, dtype=np.float32)
        self._check(load().prism_b200_project(self.h, w.handle, _p(act), int(fused), _p(out)))
        return out

    def project_device(self, weight, act_ptr, out_ptr, stream=None, fused=False):
        w = self._weight(weight)
        self._check(load().prism_b200_project_device(
            self.h, w.handle, ctypes.c_void_p(act_ptr), int(fused), ctypes.c_void_p(out_ptr),
            ctypes.c_void_p(stream) if stream else None))

    def project_f32(self, weight, x, pinned=False, out=None):
        w = self._weight(weight)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.size != w.cols:
            raise PrismB200Error(E_INVALID, "matvec requires a matching activation vector")
        if out is None:
            out = np.zeros(w.rows, dtype=np.float32)
        assert out.dtype == np.float32 and out.size == w.rows and out.flags.c_contiguous
        self._check(load().prism_b200_project_f32(self.h, w.handle, _p(x), int(pinned), _p(out)))
        return out

    def project_f32_tokens(self, weight, x, pinned=False):
        """Y[t] = W x[t] for a tile of tokens x [tokens][cols] (reference
        src/kernels/projection.rs:137-153), on the tensor cores."""
        w = self._weight(weight)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != w.cols:
            raise PrismB200Error(E_INVALID, "token tile must be [tokens][cols]")
        out = np.zeros((x.shape[0], w.rows), dtype=np.float32)
        self._check(load().prism_b200_project_f32_tokens(self.h, w.handle, x.shape[0], _p(x),
                                                         int(pinned), _p(out)))
        return out

    def project_f32_tokens_device(self, weight, tokens, x_ptr, out_ptr, pinned=False,
                                  stream=None):
        w = self._weight(weight)
        self._check(load().prism_b200_project_f32_tokens_device(
            self.h, w.handle, tokens, ctypes.c_void_p(x_ptr), int(pinned),
            ctypes.c_void_p(out_ptr), ctypes.c_void_p(stream) if stream else None))

    def project_f32_group(self, weights, x, pinned=False):
        ws = [self._weight(w) for w in weights]
        x = np.ascontiguousarray(x, dtype=np.float32)
        outs = [np.zeros(w.rows, dtype=np.float32) for w in ws]
        wh = (ctypes.c_void_p * len(ws))(*[w.handle.value for w in ws])
        oh = (ctypes.c_void_p * len(ws))(*[o.ctypes.data for o in outs])
        self._check(load().prism_b200_project_f32_group(self.h, len(ws), wh, _p(x), int(pinned), oh))
        return outs

    def project_q8(self, weight, activation, pinned=False):
        """Q8_0 activations, cols/32 Q8_DTYPE blocks (reference
        src/kernels/projection.rs:62-90): PTQ1 and PQ2 weights."""
        w = self._weight(weight)
        act = np.ascontiguousarray(activation)
        if act.dtype == Q8_DTYPE and act.size * 32 != w.cols:
            raise PrismB200Error(E_INVALID, "activation extent differs from weight columns")
        out = np.zeros(w.rows, dtype=np.float32)
        self._check(load().prism_b200_project_q8(self.h, w.handle, _p(act), int(pinned), _p(out)))
        return out

    def _tokens_group(self, fn, weights, x, pinned):
        ws = [self._weight(w) for w in weights]
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != ws[0].cols:
            raise PrismB200Error(E_INVALID, "token tile must be [tokens][cols]")
        outs = [np.zeros((x.shape[0], w.rows), dtype=np.float32) for w in ws]
        wh = (ctypes.c_void_p * len(ws))(*[w.handle.value for w in ws])
        self._check(fn(self.h, wh, x.shape[0], _p(x), int(pinned), *[_p(o) for o in outs]))
        return outs

    def project_f32_pair_tokens(self, weights, x, pinned=False):
        """Two siblings over a token tile (reference projection.rs:158-181)."""
        assert len(weights) == 2
        return self._tokens_group(load().prism_b200_project_f32_pair_tokens, weights, x, pinned)

    def project_f32_triple_tokens(self, weights, x, pinned=False):
        """Three siblings over a token tile (reference projection.rs:183-210)."""
        assert len(weights) == 3
        return self._tokens_group(load().prism_b200_project_f32_triple_tokens, weights, x, pinned)

    def project_f32_ffn_swiglu(self, gate, up, x, pinned=False):
        """up(x) * silu(gate(x)) for one token (reference projection.rs:218-234)."""
        g, u = self._weight(gate), self._weight(up)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(u.rows, dtype=np.float32)
        self._check(load().prism_b200_project_f32_ffn_swiglu(self.h, g.handle, u.handle, _p(x),
                                                             int(pinned), _p(out)))
        return out

    def project_f32_ffn_swiglu_tokens(self, gate, up, x, pinned=False):
        """up(x) * silu(gate(x)) over a token tile (reference projection.rs:236-260)."""
        g, u = self._weight(gate), self._weight(up)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros((x.shape[0], u.rows), dtype=np.float32)
        self._check(load().prism_b200_project_f32_ffn_swiglu_tokens(
            self.h, g.handle, u.handle, x.shape[0], _p(x), int(pinned), _p(out)))
        return out

    def project_f32_ffn_chain(self, gate, up, down, x, residual=None, hadamard_block_size=0,
                              pinned=False):
        """residual + down(SwiGLU(gate(x), up(x))) for one token (reference
        projection.rs:276-293)."""
        g, u, d = self._weight(gate), self._weight(up), self._weight(down)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(d.rows, dtype=np.float32)
        r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        self._check(load().prism_b200_project_f32_ffn_chain(
            self.h, g.handle, u.handle, d.handle, _p(x), _p(r) if r is not None else None,
            int(hadamard_block_size), int(pinned), _p(out)))
        return out

    def quantize_q8k(self, x, pinned=False):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.size // 256, dtype=Q8K_DTYPE)
        self._check(load().prism_b200_quantize_q8k(self.h, _p(x), x.size, int(pinned), _p(out)))
        return out

    def quantize_q8k_device(self, x_ptr, n, out_ptr, pinned=False, stream=None):
        self._check(load().prism_b200_quantize_q8k_device(
            self.h, ctypes.c_void_p(x_ptr), n, int(pinned), ctypes.c_void_p(out_ptr),
            ctypes.c_void_p(stream) if stream else None))

    def block_dots(self, weight, activation):
        w = self._weight(weight)
        act = np.ascontiguousarray(activation, dtype=Q8K_DTYPE)
        nb = w.cols // 256
        ints = np.zeros((w.rows, nb), dtype=np.int32)
        ints2 = np.zeros((w.rows, nb), dtype=np.int32)
        self._check(load().prism_b200_block_dots(self.h, w.handle, _p(act), _p(ints), _p(ints2)))
        return ints if w.kind == KIND_TQ2_0 else (ints, ints2)


def _declare_gdn(L):
    if getattr(L, "_gdn_declared", False):
        return
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    L.prism_b200_gdn_decode_device.restype = i32
    L.prism_b200_gdn_decode_device.argtypes = [vp, i32, i32, i32, i32] + [vp] * 8
    L.prism_b200_gdn_prefill_device.restype = i32
    L.prism_b200_gdn_prefill_device.argtypes = [vp, i32, i32, i32, i32, i32, i32] + [vp] * 8
    L.prism_b200_gdn_prefill_device_noalloc.restype = i32
    L.prism_b200_gdn_prefill_device_noalloc.argtypes = [vp, i32, i32, i32, i32, i32, i32] + [vp] * 8
    L.prism_b200_gdn_prefill_pinned_device.restype = i32
    L.prism_b200_gdn_prefill_pinned_device.argtypes = [vp, i32, i32, i32, i32, i32] + [vp] * 8
    L._gdn_declared = True


def gdn_decode_device(ex, batch, heads, key_heads, state, q, k, v, decay, beta, out, stream=None,
                      d=128):
    """One Gated DeltaNet step over device buffers (integer pointers)."""
    L = load()
    _declare_gdn(L)
    ex._check(L.prism_b200_gdn_decode_device(ex.h, batch, heads, key_heads, d, state, q, k, v,
                                             decay, beta, out, stream))


def gdn_prefill_device(ex, batch, tokens, heads, key_heads, chunk, state, q, k, v, decay, beta,
                       out, stream=None, d=128):
    """Chunked Gated DeltaNet prefill over device buffers."""
    L = load()
    _declare_gdn(L)
    ex._check(L.prism_b200_gdn_prefill_device(ex.h, batch, tokens, heads, key_heads, d, chunk,
                                              state, q, k, v, decay, beta, out, stream))


def gdn_prefill_pinned_device(ex, batch, tokens, heads, key_heads, state, q, k, v, decay, beta,
                              out, stream=None, d=128):
    """The reference's pinned (Swift) GDN recurrence over device buffers,
    token by token (prism_b200_gdn_prefill_pinned_device)."""
    L = load()
    _declare_gdn(L)
    ex._check(L.prism_b200_gdn_prefill_pinned_device(ex.h, batch, tokens, heads, key_heads, d,
                                                     state, q, k, v, decay, beta, out, stream))


class GdnOp(ctypes.Structure):
    """prism_b200_gdn_op: geometry of the batched gated-delta op."""
    _fields_ = [(n, ctypes.c_uint32) for n in ("width", "heads", "tokens", "sequences",
                                               "q_heads", "k_heads", "q_sequences",
                                               "k_sequences", "gate_width", "snapshots")] + \
               [("raw", ctypes.c_int32), ("replay", ctypes.c_int32),
                ("state_rows", ctypes.c_uint32), ("record_banks", ctypes.c_uint32),
                ("record_bank_elems", ctypes.c_uint64), ("records_len", ctypes.c_uint64)]


def gdn_delta_values_outputs(op):
    L = load()
    L.prism_b200_gdn_delta_values_outputs.restype = ctypes.c_size_t
    L.prism_b200_gdn_delta_values_outputs.argtypes = [ctypes.c_void_p]
    return L.prism_b200_gdn_delta_values_outputs(ctypes.byref(op))


def gdn_delta_values_device(ex, op, q, k, v, gate, beta, table, out, rows=None, bias=None,
                            weight=None, records=None, control=None, stream=None):
    """The reference's gated-delta backend op (src/backend/gdn.rs:24-300) over
    device pointers (0 / None for absent inputs)."""
    L = load()
    fn = L.prism_b200_gdn_delta_values_device
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 15
    ex._check(fn(ex.h, ctypes.byref(op), q, k, v, gate, beta, table, rows, bias, weight,
                 records, control, out, stream))


# Size of the fixed scratch of gdn_prefill_device_noalloc (include/prism_b200.h).
GDN_STATIC_SCRATCH_BYTES = 34 * 1024 * 1024


def gdn_prefill_device_noalloc(ex, batch, tokens, heads, key_heads, chunk, state, q, k, v, decay,
                               beta, out, stream=None, d=128):
    """gdn_prefill_device without any device allocation: its scratch is a
    fixed array of GDN_STATIC_SCRATCH_BYTES, shared by all callers on the
    device (overlapping calls race)."""
    L = load()
    _declare_gdn(L)
    ex._check(L.prism_b200_gdn_prefill_device_noalloc(ex.h, batch, tokens, heads, key_heads, d,
                                                      chunk, state, q, k, v, decay, beta, out,
                                                      stream))


FFN_EXCHANGE_HANDLE_BYTES = 64


class FfnChain:
    """The FFN chain over token tiles (reference src/kernels/projection.rs:
    261-350 project_f32_ffn_chain_tokens, no Hadamard): out = residual +
    down(SwiGLU(gate(x), up(x))) for [tokens][H] activations.

    tp_size > 1 makes this rank `tp_rank` of a tensor-parallel chain (one
    process and GPU per rank): gather every rank's `exchange_handle()` in rank
    order, pass the list to `connect()`, then call with the same token counts
    on every rank."""

    def __init__(self, executor, gate, up, down, max_tokens, tp_rank=0, tp_size=1):
        self.ex = executor
        ws = [executor._weight(w) for w in (gate, up, down)]
        self.H, self.F = ws[0].cols, ws[0].rows
        self.h = ctypes.c_void_p()
        executor._check(load().prism_b200_ffn_create(
            executor.h, ws[0].handle, ws[1].handle, ws[2].handle, max_tokens, tp_rank, tp_size,
            ctypes.byref(self.h)))

    def exchange_handle(self):
        buf = ctypes.create_string_buffer(FFN_EXCHANGE_HANDLE_BYTES)
        self.ex._check(load().prism_b200_ffn_exchange_handle(self.h, buf))
        return buf.raw

    def connect(self, handles):
        blob = b"".join(handles)
        self.ex._check(load().prism_b200_ffn_connect(self.h, blob))

    def __call__(self, x, residual=None, pinned=False):
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != self.H:
            raise PrismB200Error(E_INVALID, "token tile must be [tokens][hidden]")
        r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        out = np.zeros_like(x)
        self.ex._check(load().prism_b200_ffn_chain_tokens(
            self.h, x.shape[0], _p(x), _p(r) if r is not None else None, int(pinned), _p(out)))
        return out

    def device(self, tokens, x_ptr, residual_ptr, out_ptr, pinned=False, stream=None):
        self.ex._check(load().prism_b200_ffn_chain_tokens_device(
            self.h, tokens, ctypes.c_void_p(x_ptr),
            ctypes.c_void_p(residual_ptr) if residual_ptr else None, int(pinned),
            ctypes.c_void_p(out_ptr), ctypes.c_void_p(stream) if stream else None))

    def close(self):
        if self.h:
            load().prism_b200_ffn_destroy(self.h)
            self.h = None
