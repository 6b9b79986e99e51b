"""Seeded synthetic inputs with the benchmark configurations' shapes.

The reference has no public dataset for this path; these generators stand in
for real weights with the value distributions the benchmark configurations
name (uniform ternary codes, fp16 block scales in U(0.01, 0.05), N(0, 1)
activations).  numpy's PCG64 generator makes them reproducible from a seed
on any host.
"""
import numpy as np

TQ2_BLOCK = 66
Q2K_BLOCK = 84

# element i of a 256-element block -> (byte, shift) inside the 64 quant bytes
_I = np.arange(256)
_BYTE = (_I // 128) * 32 + (_I % 32)
_SHIFT = 2 * ((_I % 128) // 32)


def pack_codes(codes):
    """codes: (..., 256) uint8 in 0..3 -> (..., 64) packed bytes."""
    codes = np.asarray(codes, dtype=np.uint8)
    out = np.zeros(codes.shape[:-1] + (64,), dtype=np.uint8)
    for j in range(4):
        sel = _SHIFT == 2 * j
        out[..., _BYTE[sel]] |= (codes[..., sel] << (2 * j)).astype(np.uint8)
    return out


def tq2_weights(rows, cols, seed=0, scale_lo=0.01, scale_hi=0.05):
    """TQ2_0 rows: codes = w + 1 with w uniform in {-1, 0, +1}; one fp16
    scale per 256-block from U(scale_lo, scale_hi).  Returns uint8
    (rows, cols/256*66) in the reference byte layout."""
    assert cols % 256 == 0
    nb = cols // 256
    rng = np.random.default_rng(seed)
    out = np.empty((rows, nb, TQ2_BLOCK), dtype=np.uint8)
    step = max(1, (1 << 22) // cols)  # bound temporary memory for big matrices
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        codes = rng.integers(0, 3, size=(r1 - r0, nb, 256), dtype=np.uint8)
        out[r0:r1, :, :64] = pack_codes(codes)
        d = rng.uniform(scale_lo, scale_hi, size=(r1 - r0, nb)).astype(np.float16)
        out[r0:r1, :, 64:66] = d.view(np.uint8).reshape(r1 - r0, nb, 2)
    return out.reshape(rows, nb * TQ2_BLOCK)


def q2k_weights(rows, cols, seed=0):
    """Q2_K rows: 2-bit quants uniform in 0..3, 4-bit scales and mins
    uniform in 0..15, fp16 d ~ U(0.01, 0.05), dmin ~ U(0.005, 0.02)."""
    assert cols % 256 == 0
    nb = cols // 256
    rng = np.random.default_rng(seed)
    out = np.empty((rows, nb, Q2K_BLOCK), dtype=np.uint8)
    step = max(1, (1 << 22) // cols)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        n = r1 - r0
        out[r0:r1, :, :16] = rng.integers(0, 256, size=(n, nb, 16), dtype=np.uint8)
        out[r0:r1, :, 16:80] = pack_codes(rng.integers(0, 4, size=(n, nb, 256), dtype=np.uint8))
        d = rng.uniform(0.01, 0.05, size=(n, nb)).astype(np.float16)
        m = rng.uniform(0.005, 0.02, size=(n, nb)).astype(np.float16)
        out[r0:r1, :, 80:82] = d.view(np.uint8).reshape(n, nb, 2)
        out[r0:r1, :, 82:84] = m.view(np.uint8).reshape(n, nb, 2)
    return out.reshape(rows, nb * Q2K_BLOCK)


def activations(n, seed=0):
    """n values ~ N(0, 1), float32."""
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)
