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


def synthetic_weights(cfg, seed=0):
    """Random-init weights of the architecture: dict name -> array.  Packed
    linear weights are uint8 (rows, cols/256*block) in the reference layout;
    norms have gain 1.0; ssm_a = -1, ssm_dt.bias = 0; conv1d ~ U(-0.5, 0.5)."""
    W = {}
    kind = cfg.weight_kind

    def packed(name, rows, cols):
        W[name] = pb.synth_weights(kind, rows, cols, seed, _stream(name))

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
