"""Seeded input generators shared by the fixture script and the tests.

All streams are numpy ``Generator(PCG64(seed))``, which is bit-reproducible
across platforms, so fixtures store only reference *outputs*.
"""
from __future__ import annotations

import numpy as np

CODEBOOK_DIMS = (32, 64, 128, 256)
ROTATION_CASES = ((32, 42), (64, 0), (64, 42), (64, 55), (128, 42), (128, 55),
                  (128, 42 + 13 * 31), (128, 42 + 13 * 47), (256, 42))
EDGE_CASES = ((64, 3), (128, 2), (128, 3), (128, 4), (128, 6), (128, 8), (32, 4),
              (64, 1))

INCREMENTAL = dict(num_layers=4, B=2, H=2, D=64, key_bits=4, value_bits=2,
                   residual_window=8, protected_layers=1, max_seq_len=64,
                   layers=(0, 1), prefill=20, decode_steps=6)

BF16_CASE = dict(B=2, Hkv=2, Hq=8, D=128, T=200, key_bits=4, value_bits=2)


def to_bf16_values(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def edge_values(boundaries: np.ndarray, d: int, seed: int) -> np.ndarray:
    """Values that probe bucketize at and around every boundary."""
    b = boundaries.astype(np.float32)
    up = np.nextafter(b, np.float32(np.inf))
    dn = np.nextafter(b, np.float32(-np.inf))
    rng = np.random.Generator(np.random.PCG64(seed))
    rand = (rng.standard_normal(4096) / np.sqrt(d)).astype(np.float32)
    special = np.array([0.0, -0.0, 1.0, -1.0, 3.0e38, -3.0e38, 1e-30, -1e-30],
                       np.float32)
    y = np.concatenate([b, up, dn, special, rand]).astype(np.float32)
    pad = (-y.size) % d
    y = np.concatenate([y, np.zeros(pad, np.float32)])
    return y.reshape(-1, d)


def outlier_normal(rng, shape, n_outlier: int, scale: float) -> np.ndarray:
    """N(0,1) with `n_outlier` fixed channels per head scaled by `scale`.

    shape = (B, H, T, D); the channel set is drawn once per head.
    """
    x = rng.standard_normal(shape, dtype=np.float32)
    B, H, T, D = shape
    for h in range(H):
        ch = rng.permutation(D)[:n_outlier]
        x[:, h, :, ch] *= np.float32(scale)
    return x


def config1_inputs():
    """B1, Hq16, Hkv4, D64, T512, fp32 K/V ~ N(0,1) with 4 outlier channels x10."""
    rng = np.random.Generator(np.random.PCG64(0))
    k = outlier_normal(rng, (1, 4, 512, 64), 4, 10.0)
    v = outlier_normal(rng, (1, 4, 512, 64), 4, 10.0)
    q = rng.standard_normal((1, 16, 1, 64), dtype=np.float32)
    return k, v, q


def incremental_inputs(layer: int):
    s = INCREMENTAL
    rng = np.random.Generator(np.random.PCG64(1000 + layer))
    shape = (s["B"], s["H"], s["prefill"] + s["decode_steps"], s["D"])
    k = rng.standard_normal(shape, dtype=np.float32)
    v = rng.standard_normal(shape, dtype=np.float32)
    chunks = [(k[:, :, : s["prefill"]].copy(), v[:, :, : s["prefill"]].copy())]
    for t in range(s["prefill"], shape[2]):
        chunks.append((k[:, :, t : t + 1].copy(), v[:, :, t : t + 1].copy()))
    return chunks


def bf16_case_inputs():
    s = BF16_CASE
    rng = np.random.Generator(np.random.PCG64(7))
    k = outlier_normal(rng, (s["B"], s["Hkv"], s["T"], s["D"]), 2, 8.0)
    v = outlier_normal(rng, (s["B"], s["Hkv"], s["T"], s["D"]), 2, 8.0)
    q = rng.standard_normal((s["B"], s["Hq"], 1, s["D"]), dtype=np.float32)
    return to_bf16_values(k), to_bf16_values(v), to_bf16_values(q)
