"""Seeded synthetic GGUF blocks and activations for tests and benchmarks.

There are no real checkpoints on the target machines, so every workload is
generated from ``np.random.default_rng(seed)`` with the value distributions
the benchmark configurations name:

* Q4_K: fp16 ``d``/``dmin`` ~ |N(0, 0.02)|, 6-bit scales and mins uniform
  0..63 packed with the GGML K-quant rule, 4-bit quants uniform 0..15.
* Q6_K: int8 scales uniform -32..31, 6-bit quants uniform, fp16 d ~ |N(0, 0.01)|.
* Q8_0: fp16 d ~ |N(0, 0.005)|, int8 quants uniform -127..127.
* Q4_0 / Q5_K: random bytes with finite fp16 scales (optional types).

The block byte layouts are those of ``engine/dequant.py`` in the reference
(Q4_K :97-120, Q5_K :122-144, Q6_K :146-167, Q8_0 :75-78, Q4_0 :62-66).
"""
from __future__ import annotations

import numpy as np

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 8, 12, 13, 14
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


def row_bytes(t, cols):
    vals, nbytes = BLOCK[t]
    if cols % vals:
        raise ValueError(f'cols={cols} is not a multiple of the block size {vals}')
    return (cols // vals) * nbytes


def pack_k_scales(sc, mn):
    """Inverse of the Q4_K/Q5_K 6-bit scale/min unpacking (12 bytes per block)."""
    sc = np.asarray(sc, np.uint8)
    mn = np.asarray(mn, np.uint8)
    s = np.empty(sc.shape[:-1] + (12,), np.uint8)
    s[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = mn[..., 0:4] | ((mn[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 15) | ((mn[..., 4:8] & 15) << 4)
    return s


def _f16_bytes(values):
    return np.asarray(values, np.float16).view(np.uint8).reshape(-1, 2)


def q4_k(rng, rows, cols, d_sigma=0.02, zero_tail_cols=0):
    """Q4_K matrix [rows, cols]; the last ``zero_tail_cols`` columns decode to 0.

    ``zero_tail_cols`` implements the K padding of a matrix whose logical
    width is not a multiple of 256 (e.g. 1408 -> 1536): the padded sub-blocks
    get scale = min = 0 and quants 0, which decodes to exactly 0.0.
    """
    nb = cols // 256
    assert nb * 256 == cols
    blocks = np.empty((rows, nb, 144), np.uint8)
    blocks[:, :, 0:2] = _f16_bytes(np.abs(rng.normal(0, d_sigma, rows * nb))).reshape(rows, nb, 2)
    blocks[:, :, 2:4] = _f16_bytes(np.abs(rng.normal(0, d_sigma, rows * nb))).reshape(rows, nb, 2)
    sc = rng.integers(0, 64, size=(rows, nb, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(rows, nb, 8), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(rows, nb, 128), dtype=np.uint8)
    if zero_tail_cols:
        assert zero_tail_cols % 32 == 0 and zero_tail_cols < 256
        nsub = zero_tail_cols // 32
        sc[:, -1, 8 - nsub:] = 0
        mn[:, -1, 8 - nsub:] = 0
        for g in range(8 - nsub, 8):
            chunk = qs[:, -1, (g // 2) * 32:(g // 2 + 1) * 32]
            chunk &= np.uint8(0xF0 if g % 2 == 0 else 0x0F)
    blocks[:, :, 4:16] = pack_k_scales(sc, mn)
    blocks[:, :, 16:144] = qs
    return blocks.reshape(-1).tobytes()


def q6_k(rng, rows, cols, d_sigma=0.01):
    nb = cols // 256
    assert nb * 256 == cols
    blocks = np.empty((rows, nb, 210), np.uint8)
    blocks[:, :, 0:192] = rng.integers(0, 256, size=(rows, nb, 192), dtype=np.uint8)
    blocks[:, :, 192:208] = rng.integers(-32, 32, size=(rows, nb, 16)).astype(np.int8).view(np.uint8)
    blocks[:, :, 208:210] = _f16_bytes(np.abs(rng.normal(0, d_sigma, rows * nb))).reshape(rows, nb, 2)
    return blocks.reshape(-1).tobytes()


def q8_0(rng, rows, cols, d_sigma=0.005):
    nb = cols // 32
    assert nb * 32 == cols
    blocks = np.empty((rows, nb, 34), np.uint8)
    blocks[:, :, 0:2] = _f16_bytes(np.abs(rng.normal(0, d_sigma, rows * nb))).reshape(rows, nb, 2)
    blocks[:, :, 2:34] = rng.integers(-127, 128, size=(rows, nb, 32)).astype(np.int8).view(np.uint8)
    return blocks.reshape(-1).tobytes()


def random_blocks(rng, t, rows, cols, d=0.03125, dmin=0.015625):
    """Reference-test style: uniform random bytes, then fixed fp16 scale fields.

    Mirrors the fixtures of tests/test_dequant.py:119-230 in the reference
    (random block bytes with ``d`` overwritten by a constant).
    """
    vals, nbytes = BLOCK[t]
    nb = cols // vals
    blocks = rng.integers(0, 256, size=(rows, nb, nbytes), dtype=np.uint8)
    doff = 208 if t == Q6_K else 0
    blocks[:, :, doff:doff + 2] = np.frombuffer(np.float16(d).tobytes(), np.uint8)
    if t in (Q4_K, Q5_K):
        blocks[:, :, 2:4] = np.frombuffer(np.float16(dmin).tobytes(), np.uint8)
    return blocks.reshape(-1).tobytes()


def make(rng, t, rows, cols):
    """Benchmark-distribution generator for any supported type."""
    if t == Q4_K:
        return q4_k(rng, rows, cols)
    if t == Q6_K:
        return q6_k(rng, rows, cols)
    if t == Q8_0:
        return q8_0(rng, rows, cols)
    return random_blocks(rng, t, rows, cols, d=0.0005, dmin=0.00025)
