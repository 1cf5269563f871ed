"""TEST INFRASTRUCTURE ONLY - random legal GGML blocks and a float64 dequantiser.

``random_blocks`` follows the reference tests' recipe for exercising every
bit of a packed format (qwen/test_cpu_dispatch.py:19-33,
qwen/test_gpu.py:121-128): uniformly random bytes with the fp16 scale fields
overwritten by fixed small scales, so decoded weights stay finite and small.

``dequant64`` is an independent NumPy expansion of the two formats on the
hot path (Q4_K, IQ4_NL) plus F32, written from the GGML block layouts, used
as a float64 cross-check next to the reference's own ``qwen/quant.py``.
"""
from __future__ import annotations

import numpy as np

FORMATS = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 6: (32, 22), 7: (32, 24), 8: (32, 34),
           12: (256, 144), 13: (256, 176), 14: (256, 210), 20: (32, 18)}
IQ4NL = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float64)


def row_bytes(typ: int, cols: int) -> int:
    block, size = FORMATS[typ]
    if cols % block:
        raise ValueError("block does not divide the row")
    return cols // block * size


def random_blocks(rng: np.random.Generator, typ: int, rows: int, cols: int,
                  d: float = 0.0005, dmin: float = 0.0002) -> np.ndarray:
    """[rows, row_bytes] uint8 of random legal blocks of GGML type ``typ``."""
    if typ == 0:
        return rng.normal(0, 0.05, (rows, cols)).astype("<f4").view(np.uint8).reshape(rows, -1)
    if typ == 1:
        return rng.normal(0, 0.05, (rows, cols)).astype("<f2").view(np.uint8).reshape(rows, -1)
    if typ == 30:
        bits = (rng.normal(0, 0.05, (rows, cols)).astype("<f4").view("<u4") >> 16).astype("<u2")
        return bits.view(np.uint8).reshape(rows, -1)
    block, size = FORMATS[typ]
    data = rng.integers(0, 256, (rows, cols // block, size), dtype=np.uint8)
    off = 208 if typ == 14 else 0
    data[..., off:off + 2] = np.array([d], "<f2").view(np.uint8)
    if typ in (7, 12, 13):
        data[..., 2:4] = np.array([dmin], "<f2").view(np.uint8)
    return data.reshape(rows, -1)


def dequant64(packed: np.ndarray, typ: int, rows: int, cols: int) -> np.ndarray:
    """Float64 values of a packed [rows, row_bytes] matrix (types 0, 12, 20)."""
    p = np.ascontiguousarray(packed).reshape(rows, -1)
    if typ == 0:
        return p.view("<f4").astype(np.float64).reshape(rows, cols)
    if typ == 20:
        b = p.reshape(rows, cols // 32, 18)
        d = b[..., 0:2].copy().view("<f2").astype(np.float64)  # [rows, nb, 1]
        q = b[..., 2:18]
        codes = np.concatenate([q & 15, q >> 4], axis=-1)  # value j: byte j%16, nibble j//16
        return (IQ4NL[codes] * d).reshape(rows, cols)
    if typ == 12:
        b = p.reshape(rows, cols // 256, 144)
        d = b[..., 0:2].copy().view("<f2").astype(np.float64)
        dmin = b[..., 2:4].copy().view("<f2").astype(np.float64)
        sc = b[..., 4:16].astype(np.int64)
        s = np.empty(sc.shape[:-1] + (8,), np.int64)
        m = np.empty_like(s)
        for g in range(8):
            if g < 4:
                s[..., g] = sc[..., g] & 63
                m[..., g] = sc[..., g + 4] & 63
            else:
                s[..., g] = (sc[..., g + 4] & 15) | ((sc[..., g - 4] >> 6) << 4)
                m[..., g] = (sc[..., g + 4] >> 4) | ((sc[..., g] >> 6) << 4)
        qs = b[..., 16:144].reshape(rows, cols // 256, 4, 32)
        q = np.stack([qs & 15, qs >> 4], axis=-2).reshape(rows, cols // 256, 8, 32).astype(np.float64)
        w = q * (d * s)[..., None] - (dmin * m)[..., None]
        return w.reshape(rows, cols)
    raise ValueError(f"dequant64 covers types 0, 12, 20, not {typ}")
