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
        "po_tq2_decode": (i32, [vp, sz, vp]),
        "po_tq2_quantize": (i32, [vp, sz, vp]),
        "po_tq2_block_dots": (i32, [vp, vp, sz, vp]),
        "po_tq2_dot": (i32, [vp, vp, sz, vp]),
        "po_q2k_decode": (i32, [vp, sz, vp]),
        "po_q2k_block_dots": (i32, [vp, vp, sz, vp, vp]),
        "po_q2k_dot": (i32, [vp, vp, sz, vp]),
        "po_matvec": (i32, [u32, vp, sz, sz, vp, vp, i32]),
        "po_float_dot": (f32, [vp, vp, sz]),
        "po_f16_dot": (f32, [vp, vp, sz]),
        "po_silu": (f32, [f32]),
        "po_sigmoid": (f32, [f32]),
        "po_recurrent_decay": (i32, [f32, f32, f32, vp]),
        "po_rms_norm": (i32, [vp, vp, sz, f32, vp]),
        "po_add_rms_norm": (i32, [vp, vp, vp, sz, f32, vp]),
        "po_l2_norm": (None, [vp, sz, f32]),
        "po_softmax_round_f16": (i32, [vp, sz]),
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


def block_bytes(kind):
    return {35: 66, 10: 84}[kind]


def decode(kind, packed):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    nb = packed.size // block_bytes(kind)
    out = np.zeros(nb * 256, dtype=np.float32)
    fn = lib().po_tq2_decode if kind == 35 else lib().po_q2k_decode
    _check(fn(_p(packed), nb, _p(out)))
    return out


def tq2_quantize(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 256 * 66, dtype=np.uint8)
    _check(lib().po_tq2_quantize(_p(x), x.size, _p(out)))
    return out


def dot(kind, packed_row, act):
    packed_row = np.ascontiguousarray(packed_row, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    out = np.zeros(1, dtype=np.float32)
    fn = lib().po_tq2_dot if kind == 35 else lib().po_q2k_dot
    _check(fn(_p(packed_row), _p(act), act.size, _p(out)))
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


def matvec(kind, weights, rows, cols, act, threads=1):
    weights = np.ascontiguousarray(weights, dtype=np.uint8)
    act = np.ascontiguousarray(act, dtype=Q8K_DTYPE)
    y = np.zeros(rows, dtype=np.float32)
    _check(lib().po_matvec(kind, _p(weights), rows, cols, _p(act), _p(y), threads))
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


def recurrent_decay(alpha, time_bias, decay_weight):
    out = np.zeros(1, dtype=np.float32)
    _check(lib().po_recurrent_decay(alpha, time_bias, decay_weight, _p(out)))
    return out[0]
