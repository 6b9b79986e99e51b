"""Qwen3.5-style hybrid decoder geometry and seeded synthetic weights.

Geometry keys mirror the reference's GGUF metadata (reference
src/graph.rs:2966-3056: ``qwen35.embedding_length``, ``block_count``,
``attention.head_count`` ...); tensor names mirror its tensor binding
(src/graph.rs:3112-3238).  Every ``full_interval``-th layer
(``(i + 1) % full_interval == 0``) is gated full attention; the others are
Gated DeltaNet.  The output head is tied to ``token_embd.weight``.
"""
import zlib
from dataclasses import dataclass, field, replace

import numpy as np

import prism_b200 as pb


@dataclass(frozen=True)
class Qwen35Config:
    hidden: int = 2560
    layers: int = 32
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 256
    rope_dim: int = 64
    rope_sections: tuple = (11, 11, 10, 0)
    rope_base: float = 1.0e7
    eps: float = 1.0e-6
    ffn: int = 9216
    vocab: int = 151936
    ssm_state: int = 128
    ssm_groups: int = 16
    ssm_values: int = 16
    conv_kernel: int = 4
    full_interval: int = 4
    context: int = 1024
    weight_kind: int = pb.KIND_TQ2_0

    def is_full(self, layer):
        return (layer + 1) % self.full_interval == 0

    @property
    def key_width(self):
        return self.ssm_state * self.ssm_groups

    @property
    def value_width(self):
        return self.ssm_state * self.ssm_values

    @property
    def conv_channels(self):
        return 2 * self.key_width + self.value_width

    def linear_shapes(self, layer):
        """(name suffix, rows, cols) of every packed weight of a layer."""
        h, hd = self.hidden, self.head_dim
        out = [("ffn_gate.weight", self.ffn, h), ("ffn_up.weight", self.ffn, h),
               ("ffn_down.weight", h, self.ffn)]
        if self.is_full(layer):
            out += [("attn_q.weight", self.heads * hd * 2, h),
                    ("attn_k.weight", self.kv_heads * hd, h),
                    ("attn_v.weight", self.kv_heads * hd, h),
                    ("attn_output.weight", h, self.heads * hd)]
        else:
            out += [("attn_qkv.weight", self.conv_channels, h),
                    ("attn_gate.weight", self.value_width, h),
                    ("ssm_beta.weight", self.ssm_values, h),
                    ("ssm_alpha.weight", self.ssm_values, h),
                    ("ssm_out.weight", h, self.value_width)]
        return out

    def linear_bytes(self):
        """Bytes of every packed weight once, the tied LM head included."""
        bb = pb.BLOCK_BYTES[self.weight_kind]
        total = self.vocab * self.hidden // 256 * bb
        for l in range(self.layers):
            for _, rows, cols in self.linear_shapes(l):
                total += rows * cols // 256 * bb
        return total

    def weight_bytes_per_token(self, context=0):
        """Algorithmic HBM bytes of one decode token: every packed weight
        once (LM head included), recurrent state read + write, conv state
        read + write, and the binary16 KV cache read at `context` tokens."""
        bb = pb.BLOCK_BYTES[self.weight_kind]
        total = self.vocab * self.hidden // 256 * bb  # tied LM head
        total += self.hidden // 256 * bb  # embedding row
        for l in range(self.layers):
            for _, rows, cols in self.linear_shapes(l):
                total += rows * cols // 256 * bb
            if self.is_full(l):
                total += 2 * context * self.kv_heads * self.head_dim * 2
            else:
                total += 2 * self.ssm_values * self.ssm_state * self.ssm_state * 4
                total += 2 * self.conv_channels * (self.conv_kernel - 1) * 4
        return total


CONFIG1 = Qwen35Config()
# a small geometry with the same structure, for fast full-sequence parity
SMALL = Qwen35Config(hidden=512, layers=4, heads=4, kv_heads=2, head_dim=256, ffn=1024,
                     vocab=2048, ssm_state=128, ssm_groups=2, ssm_values=4, context=256)


def _stream(name):
    return zlib.crc32(name.encode())


def synthetic_weights(cfg, seed=0, generator=None):
    """Random-init weights of the architecture: dict name -> array.  Packed
    linear weights are uint8 (rows, cols/256*block) in the reference layout;
    norms have gain 1.0; ssm_a = -1, ssm_dt.bias = 0; conv1d ~ U(-0.5, 0.5).
    `generator(kind, rows, cols, seed, stream)` makes the packed weights
    (default: the library's seeded generator, prism_b200_synth_weights)."""
    W = {}
    kind = cfg.weight_kind
    gen = generator or pb.synth_weights

    def packed(name, rows, cols):
        W[name] = gen(kind, rows, cols, seed, _stream(name))

    packed("token_embd.weight", cfg.vocab, cfg.hidden)
    W["output_norm.weight"] = np.ones(cfg.hidden, np.float32)
    rng = np.random.default_rng(seed + 7)
    for l in range(cfg.layers):
        p = "blk.%d." % l
        W[p + "attn_norm.weight"] = np.ones(cfg.hidden, np.float32)
        W[p + "post_attention_norm.weight"] = np.ones(cfg.hidden, np.float32)
        for suffix, rows, cols in cfg.linear_shapes(l):
            packed(p + suffix, rows, cols)
        if cfg.is_full(l):
            W[p + "attn_q_norm.weight"] = np.ones(cfg.head_dim, np.float32)
            W[p + "attn_k_norm.weight"] = np.ones(cfg.head_dim, np.float32)
        else:
            W[p + "ssm_conv1d.weight"] = rng.uniform(
                -0.5, 0.5, (cfg.conv_channels, cfg.conv_kernel)).astype(np.float32)
            W[p + "ssm_dt.bias"] = np.zeros(cfg.ssm_values, np.float32)
            W[p + "ssm_a"] = -np.ones(cfg.ssm_values, np.float32)
            W[p + "ssm_norm.weight"] = np.ones(cfg.ssm_state, np.float32)
    return W


def prompt_tokens(cfg, n=512, seed=1):
    """Random prompt of n token ids uniform in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, cfg.vocab, n).astype(np.uint32)


class _CConfig(__import__("ctypes").Structure):
    import ctypes as _c
    _fields_ = [("hidden", _c.c_uint32), ("layers", _c.c_uint32), ("heads", _c.c_uint32),
                ("kv_heads", _c.c_uint32), ("head_dim", _c.c_uint32), ("rope_dim", _c.c_uint32),
                ("rope_sections", _c.c_uint32 * 4), ("rope_base", _c.c_float), ("eps", _c.c_float),
                ("ffn", _c.c_uint32), ("vocab", _c.c_uint32), ("ssm_state", _c.c_uint32),
                ("ssm_groups", _c.c_uint32), ("ssm_values", _c.c_uint32),
                ("conv_kernel", _c.c_uint32), ("full_interval", _c.c_uint32),
                ("context", _c.c_uint32), ("kv_policy", _c.c_uint32), ("weight_kind", _c.c_uint32)]


KV_F16, KV_Q8_0 = 0, 1
# the reference's rotated scalar policies: rsq4, rsq4vf, rsq4k3v
KV_RSQ4, KV_RSQ4VF, KV_RSQ4K3V = 2, 3, 4


def c_config(cfg, kv_policy=KV_F16):
    """The C ABI's prism_b200_qwen35_config of a Qwen35Config."""
    import ctypes as c
    cc = _CConfig()
    for f, _ in _CConfig._fields_:
        if f == "rope_sections":
            cc.rope_sections = (c.c_uint32 * 4)(*cfg.rope_sections)
        elif f == "kv_policy":
            cc.kv_policy = kv_policy
        else:
            setattr(cc, f, getattr(cfg, f))
    return cc


def config_from_c(cc):
    """A Qwen35Config of a prism_b200_qwen35_config (the inverse of c_config)."""
    kw = {}
    for f, _ in _CConfig._fields_:
        if f == "rope_sections":
            kw[f] = tuple(cc.rope_sections)
        elif f != "kv_policy":
            kw[f] = getattr(cc, f)
    return Qwen35Config(**kw)


class GgufFile:
    """A parsed GGUF file (prism_b200_gguf): the reference's Model::load
    checks; `config` is the Qwen35 geometry from its `qwen35.*` keys."""

    def __init__(self, path):
        import ctypes as c
        self.h = None
        self.L = L = pb.load()
        _declare_gguf(L)
        err = c.create_string_buffer(512)
        h = c.c_void_p()
        st = L.prism_b200_gguf_open(str(path).encode(), c.byref(h), err, len(err))
        if st:
            raise pb.PrismB200Error(st, err.value.decode())
        self.h = h

    def config(self, context, kv_policy=KV_F16):
        import ctypes as c
        cc = _CConfig()
        err = c.create_string_buffer(512)
        st = self.L.prism_b200_gguf_qwen35_config(self.h, context, kv_policy, c.byref(cc), err,
                                                  len(err))
        if st:
            raise pb.PrismB200Error(st, err.value.decode())
        return config_from_c(cc)

    def tensors(self):
        """[(name, type, dims, bytes)] in file order; bytes are a copy."""
        import ctypes as c
        out = []
        for i in range(self.L.prism_b200_gguf_tensor_count(self.h)):
            name, typ = c.c_char_p(), c.c_uint32()
            dims, nd = (c.c_uint64 * 4)(), c.c_uint32()
            data, nbytes = c.c_void_p(), c.c_uint64()
            self.L.prism_b200_gguf_tensor(self.h, i, c.byref(name), c.byref(typ), dims,
                                          c.byref(nd), c.byref(data), c.byref(nbytes))
            out.append((name.value.decode(), typ.value, list(dims)[:nd.value],
                        c.string_at(data.value, nbytes.value)))
        return out

    def close(self):
        if self.h:
            self.L.prism_b200_gguf_close(self.h)
            self.h = None

    def __del__(self):
        self.close()


def _declare_gguf(L):
    import ctypes as c
    if getattr(L, "_gguf_declared", False):
        return
    vp, sz = c.c_void_p, c.c_size_t
    for name, res, args in (
            ("prism_b200_gguf_open", c.c_int, [c.c_char_p, c.POINTER(vp), c.c_char_p, sz]),
            ("prism_b200_gguf_close", None, [vp]),
            ("prism_b200_gguf_tensor_count", c.c_int64, [vp]),
            ("prism_b200_gguf_tensor", c.c_int, [vp, sz, c.POINTER(c.c_char_p),
                                                 c.POINTER(c.c_uint32), c.POINTER(c.c_uint64),
                                                 c.POINTER(c.c_uint32), c.POINTER(vp),
                                                 c.POINTER(c.c_uint64)]),
            ("prism_b200_gguf_qwen35_config", c.c_int, [vp, c.c_uint32, c.c_uint32, vp,
                                                        c.c_char_p, sz]),
            ("prism_b200_model_load_gguf", c.c_int, [vp, vp, c.c_uint32, c.c_uint32,
                                                     c.POINTER(vp)])):
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    L._gguf_declared = True


def tp_plan(cfg, rank, size):
    """The slice of every linear rank `rank` of a `size`-way tensor-parallel
    batch owns (host only): dict of [first, end) ranges -- query heads, KV
    heads, Gated DeltaNet heads, FFN 256-row blocks, vocabulary rows, hidden
    rows of the projections leaving the heads and the FFN (exact form)."""
    import ctypes as c
    L = pb.load()
    fn = L.prism_b200_tp_plan
    fn.restype = c.c_int
    fn.argtypes = [c.c_void_p, c.c_uint32, c.c_uint32, c.c_void_p]
    cc = c_config(cfg)
    out = np.zeros(12, np.int32)
    st = fn(c.byref(cc), rank, size, out.ctypes.data)
    if st:
        raise pb.PrismB200Error(st, "tensor-parallel plan %d/%d" % (rank, size))
    keys = ["query_heads", "kv_heads", "gdn_heads", "ffn_blocks", "vocab_rows", "hidden_rows"]
    return {k: (int(out[2 * i]), int(out[2 * i + 1])) for i, k in enumerate(keys)}


def _declare_model(L):
    import ctypes as c
    vp, i32, sz, u32 = c.c_void_p, c.c_int, c.c_size_t, c.c_uint32
    for name, res, args in [
        ("prism_b200_model_create", i32, [vp, vp, c.POINTER(vp)]),
        ("prism_b200_model_destroy", None, [vp]),
        ("prism_b200_model_set_tensor", i32, [vp, c.c_char_p, vp]),
        ("prism_b200_model_set_vector", i32, [vp, c.c_char_p, vp, sz]),
        ("prism_b200_model_finalize", i32, [vp]),
        ("prism_b200_model_reset", i32, [vp]),
        ("prism_b200_model_position", c.c_int64, [vp]),
        ("prism_b200_model_persistent", i32, [vp]),
        ("prism_b200_model_evaluate", i32, [vp, u32, vp, vp]),
        ("prism_b200_model_generate", i32, [vp, vp, sz, sz, vp]),
        ("prism_b200_model_decode_async", i32, [vp, sz]),
        ("prism_b200_model_read_state", c.c_int64, [vp, u32, u32, vp, sz]),
    ]:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


class Qwen35Model:
    """The hybrid decoder on the device, through the C ABI.  Mirrors the
    reference's Decoder surface: reset, evaluate (one token -> logits),
    generate (prompt ingestion + greedy decode)."""

    def __init__(self, executor, cfg, kv_policy=KV_F16):
        import ctypes as c
        L = pb.load()
        _declare_model(L)
        self.L, self.ex, self.cfg = L, executor, cfg
        cc = c_config(cfg, kv_policy)
        self._cc = cc
        h = c.c_void_p()
        executor._check(L.prism_b200_model_create(executor.h, c.byref(cc), c.byref(h)))
        self.h = h

    @classmethod
    def from_gguf(cls, executor, gguf, context, kv_policy=KV_F16):
        """The model of a GGUF file (prism_b200_model_load_gguf): geometry
        from its metadata, every tensor bound by name, finalized."""
        import ctypes as c
        g = gguf if isinstance(gguf, GgufFile) else GgufFile(gguf)
        self = cls.__new__(cls)
        self.L, self.ex = g.L, executor
        _declare_model(self.L)
        self.cfg = g.config(context, kv_policy)
        self._cc = c_config(self.cfg, kv_policy)
        h = c.c_void_p()
        executor._check(self.L.prism_b200_model_load_gguf(executor.h, g.h, context, kv_policy,
                                                          c.byref(h)))
        self.h = h
        return self

    def close(self):
        if self.h:
            self.L.prism_b200_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, weights):
        import ctypes as c
        for name, arr in weights.items():
            if arr.dtype == np.uint8:
                rows = arr.shape[0]
                cols = arr.shape[1] // pb.BLOCK_BYTES[self.cfg.weight_kind] * 256
                t = pb.Tensor(self.cfg.weight_kind, cols, rows, arr)._c()
                st = self.L.prism_b200_model_set_tensor(self.h, name.encode(), c.byref(t))
            else:
                a = np.ascontiguousarray(arr, np.float32).reshape(-1)
                st = self.L.prism_b200_model_set_vector(self.h, name.encode(), a.ctypes.data, a.size)
            self.ex._check(st)
        self.ex._check(self.L.prism_b200_model_finalize(self.h))

    def reset(self):
        self.ex._check(self.L.prism_b200_model_reset(self.h))

    @property
    def position(self):
        return self.L.prism_b200_model_position(self.h)

    @property
    def step_mode(self):
        """2: the dataflow step kernel (the default where eligible), 0: the
        per-phase kernel sequence (PRISM_B200_STEP=seq at load)."""
        import ctypes as c
        L = self.L
        if not getattr(L, "_mode_declared", False):
            L.prism_b200_model_step_mode.restype = c.c_int
            L.prism_b200_model_step_mode.argtypes = [c.c_void_p]
            L._mode_declared = True
        return int(L.prism_b200_model_step_mode(self.h))

    @property
    def persistent(self):
        """True when each step runs as one cooperative kernel (the dataflow
        step)."""
        return bool(self.L.prism_b200_model_persistent(self.h))

    def evaluate(self, token, logits=True):
        import ctypes as c
        out = np.zeros(self.cfg.vocab, np.float32) if logits else None
        g = np.zeros(1, np.uint32)
        self.ex._check(self.L.prism_b200_model_evaluate(
            self.h, int(token), out.ctypes.data if logits else None, g.ctypes.data))
        return out, int(g[0])

    def generate(self, prompt, n_new):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(n_new, 1), np.uint32)
        self.ex._check(self.L.prism_b200_model_generate(self.h, prompt.ctypes.data, prompt.size,
                                                        n_new, out.ctypes.data))
        return out[:n_new]

    def decode_async(self, steps):
        self.ex._check(self.L.prism_b200_model_decode_async(self.h, steps))

    def read_state(self, layer, which):
        """which: 0 conv, 1 matrix, 2 keys, 3 values, 4 hidden."""
        c = self.cfg
        shapes = {0: ((c.conv_channels, c.conv_kernel - 1), np.float32),
                  1: ((c.ssm_values, c.ssm_state, c.ssm_state), np.float32),
                  2: ((self.position, c.kv_heads * c.head_dim), np.uint16),
                  3: ((self.position, c.kv_heads * c.head_dim), np.uint16),
                  4: ((c.hidden,), np.float32)}
        shape, dt = shapes[which]
        out = np.zeros(shape, dt)
        n = self.L.prism_b200_model_read_state(self.h, layer, which, out.ctypes.data, out.nbytes)
        if n < 0:
            raise pb.PrismB200Error(-n, "state readback failed")
        return out

    # -- checkpoints (reference Decoder::checkpoint / restore) --------------
    def _declare_checkpoint(self):
        import ctypes as c
        L = self.L
        if getattr(L, "_ckpt_declared", False):
            return
        vp = c.c_void_p
        for name, res, args in (
                ("prism_b200_model_checkpoint", c.c_int, [vp, c.POINTER(vp)]),
                ("prism_b200_model_checkpoint_into", c.c_int, [vp, vp]),
                ("prism_b200_model_restore", c.c_int, [vp, vp]),
                ("prism_b200_checkpoint_bytes", c.c_int64, [vp]),
                ("prism_b200_checkpoint_position", c.c_int64, [vp]),
                ("prism_b200_checkpoint_destroy", None, [vp])):
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        L._ckpt_declared = True

    def checkpoint(self):
        """A device-resident copy of the decoder state (Checkpoint)."""
        import ctypes as c
        self._declare_checkpoint()
        h = c.c_void_p()
        self.ex._check(self.L.prism_b200_model_checkpoint(self.h, c.byref(h)))
        return Checkpoint(self.L, h)

    def checkpoint_into(self, cp):
        self._declare_checkpoint()
        self.ex._check(self.L.prism_b200_model_checkpoint_into(self.h, cp.h))

    def restore(self, cp):
        self._declare_checkpoint()
        self.ex._check(self.L.prism_b200_model_restore(self.h, cp.h))

    def records(self, layer, value=False):
        """The rotated scalar KV records (kv_policy KV_RSQ4, _RSQ4VF,
        _RSQ4K3V) of a full layer: uint8 (position, kv_heads, record bytes)."""
        c = self.cfg
        bits = 3 if (value and self._cc.kv_policy == KV_RSQ4K3V) else 4
        rb = pb.kvq_record_bytes(bits)
        out = np.zeros((self.position, c.kv_heads, rb), np.uint8)
        n = self.L.prism_b200_model_read_state(self.h, layer, 3 if value else 2,
                                               out.ctypes.data, out.nbytes)
        if n < 0:
            raise pb.PrismB200Error(-n, "state readback failed")
        return out

    def step_timings(self):
        """One device-driven decode step with per-phase CUDA events:
        (attention_ms[layers], ffn_ms[layers], head_ms, total_ms)."""
        import ctypes as c
        L = self.L
        if not getattr(L, "_timings_declared", False):
            L.prism_b200_model_step_timings.restype = c.c_int
            L.prism_b200_model_step_timings.argtypes = [c.c_void_p] * 5
            L._timings_declared = True
        att = np.zeros(self.cfg.layers, np.float32)
        ffn = np.zeros(self.cfg.layers, np.float32)
        head = np.zeros(1, np.float32)
        tot = np.zeros(1, np.float32)
        self.ex._check(L.prism_b200_model_step_timings(self.h, att.ctypes.data, ffn.ctypes.data,
                                                       head.ctypes.data, tot.ctypes.data))
        return att, ffn, float(head[0]), float(tot[0])

    def stream(self):
        """The model's cudaStream_t (an integer handle)."""
        import ctypes as c
        L = self.L
        if not getattr(L, "_mstream_declared", False):
            L.prism_b200_model_stream.restype = c.c_void_p
            L.prism_b200_model_stream.argtypes = [c.c_void_p]
            L._mstream_declared = True
        return L.prism_b200_model_stream(self.h)

    def set_prompt(self, tokens):
        import ctypes as c
        L = self.L
        if not getattr(L, "_prompt_declared", False):
            L.prism_b200_model_set_prompt.restype = c.c_int
            L.prism_b200_model_set_prompt.argtypes = [c.c_void_p, c.c_void_p, c.c_size_t]
            L.prism_b200_model_ingest_async.restype = c.c_int
            L.prism_b200_model_ingest_async.argtypes = [c.c_void_p, c.c_size_t]
            L.prism_b200_model_prefill_async.restype = c.c_int
            L.prism_b200_model_prefill_async.argtypes = [c.c_void_p, c.c_size_t]
            L.prism_b200_model_ingest_block.restype = c.c_int
            L.prism_b200_model_ingest_block.argtypes = [c.c_void_p, c.c_void_p, c.c_size_t]
            L._prompt_declared = True
        t = np.ascontiguousarray(tokens, np.uint32)
        self.ex._check(L.prism_b200_model_set_prompt(self.h, t.ctypes.data, t.size))

    def ingest_async(self, n):
        """Enqueue n one-token ingestion steps of the tokens set_prompt placed."""
        self.set_prompt  # declarations
        self.ex._check(self.L.prism_b200_model_ingest_async(self.h, n))

    def prefill_async(self, n):
        """Enqueue the batched ingestion of the n tokens set_prompt placed
        (same resulting state as ingest_async(n))."""
        self.set_prompt  # declarations
        self.ex._check(self.L.prism_b200_model_prefill_async(self.h, n))

    def ingest_block(self, tokens):
        """Decoder::ingest_block: place, ingest and wait (at most
        MAX_PREFILL_BLOCK_TOKENS tokens)."""
        self.set_prompt  # declarations
        t = np.ascontiguousarray(tokens, np.uint32)
        self.ex._check(self.L.prism_b200_model_ingest_block(self.h, t.ctypes.data, t.size))


def _declare_batch(L):
    import ctypes as c
    if getattr(L, "_batch_declared", False):
        return
    vp, i32, sz, u32, u64 = c.c_void_p, c.c_int, c.c_size_t, c.c_uint32, c.c_uint64
    for name, res, args in [
        ("prism_b200_batch_create", i32, [vp, u32, u32, c.POINTER(vp)]),
        ("prism_b200_batch_destroy", None, [vp]),
        ("prism_b200_batch_reset", i32, [vp]),
        ("prism_b200_batch_step", i32, [vp, vp, vp]),
        ("prism_b200_batch_decode_async", i32, [vp, sz]),
        ("prism_b200_batch_stream", vp, [vp]),
        ("prism_b200_batch_fill_context", i32, [vp, u32, u64]),
        ("prism_b200_batch_read_state", c.c_int64, [vp, u32, u32, u32, vp, sz]),
        ("prism_b200_batch_create_tp", i32, [vp, u32, u32, u32, u32, u32, c.POINTER(vp)]),
        ("prism_b200_batch_exchange_handle", i32, [vp, vp]),
        ("prism_b200_batch_connect", i32, [vp, vp]),
    ]:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    L._batch_declared = True


EXCHANGE_HANDLE_BYTES = 64
TP_EXACT, TP_ALLREDUCE = 0, 1


class Checkpoint:
    """A decoder checkpoint on the device (prism_b200_checkpoint)."""

    def __init__(self, L, handle):
        self.L, self.h = L, handle

    @property
    def bytes(self):
        return self.L.prism_b200_checkpoint_bytes(self.h)

    @property
    def position(self):
        return self.L.prism_b200_checkpoint_position(self.h)

    def close(self):
        if self.h:
            self.L.prism_b200_checkpoint_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Qwen35Batch:
    """Batched serving over a loaded Qwen35Model's weights: `sequences`
    sequences of up to `context` positions, one token each per step.

    With tp_size > 1 this is rank `tp_rank` of a tensor-parallel batch (one
    process and GPU per rank, all stepping the same tokens): gather every
    rank's `exchange_handle()` in rank order and pass the list to
    `connect()` before the first step.  `tp_mode` TP_EXACT gathers the
    head / FFN outputs and column-splits every projection (bit-identical to
    one GPU); TP_ALLREDUCE row-splits attn_output / ssm_out / ffn_down and
    all-reduces their partial sums (matches one GPU to rounding only)."""

    def __init__(self, model, sequences, context, tp_rank=0, tp_size=1, tp_mode=TP_EXACT):
        import ctypes as c
        self.model, self.B, self.context = model, sequences, context
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.L = model.L
        _declare_batch(self.L)
        h = c.c_void_p()
        model.ex._check(self.L.prism_b200_batch_create_tp(model.h, sequences, context, tp_rank,
                                                          tp_size, tp_mode, c.byref(h)))
        self.h = h

    def exchange_handle(self):
        buf = np.zeros(EXCHANGE_HANDLE_BYTES, np.uint8)
        self.model.ex._check(self.L.prism_b200_batch_exchange_handle(self.h, buf.ctypes.data))
        return buf.tobytes()

    def connect(self, handles):
        assert len(handles) == self.tp_size
        buf = np.frombuffer(b"".join(handles), np.uint8).copy()
        assert buf.size == EXCHANGE_HANDLE_BYTES * self.tp_size
        self.model.ex._check(self.L.prism_b200_batch_connect(self.h, buf.ctypes.data))

    def step(self, tokens):
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        assert tokens.size == self.B
        out = np.zeros(self.B, np.uint32)
        self.model.ex._check(self.L.prism_b200_batch_step(self.h, tokens.ctypes.data,
                                                          out.ctypes.data))
        return out

    def decode_async(self, steps):
        self.model.ex._check(self.L.prism_b200_batch_decode_async(self.h, steps))

    @property
    def stream(self):
        return self.L.prism_b200_batch_stream(self.h)

    def fill_context(self, position, seed=0):
        self.model.ex._check(self.L.prism_b200_batch_fill_context(self.h, position, seed))

    def reset(self):
        self.model.ex._check(self.L.prism_b200_batch_reset(self.h))

    def read_state(self, seq, layer, which, nbytes=None):
        c = self.model.cfg
        sizes = {0: c.conv_channels * (c.conv_kernel - 1) * 4,
                 1: c.ssm_values * c.ssm_state * c.ssm_state * 4,
                 2: self.context * c.kv_heads * c.head_dim * 2,
                 3: self.context * c.kv_heads * c.head_dim * 2,
                 4: c.hidden * 4}
        out = np.zeros(nbytes or sizes[which], np.uint8)
        n = self.L.prism_b200_batch_read_state(self.h, seq, layer, which, out.ctypes.data,
                                               out.nbytes)
        if n < 0:
            raise pb.PrismB200Error(-n, "batch state readback failed")
        out = out[:n]
        return out.view(np.float32) if which in (0, 1, 4) else out

    def close(self):
        if self.h:
            self.L.prism_b200_batch_destroy(self.h)
            self.h = None
