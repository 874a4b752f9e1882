"""Seeded synthetic GGUF tensors and activations with the distributions of the benchmark configurations (no model
files exist here; these stand in for them). All generators return GGUF block bytes exactly as a .gguf file stores
them, row-major (rows x row_bytes uint8).

  Q4_0: fp16 d = |N(0, 0.02)|, 4-bit quants uniform in 0..15                    (config 0, 3, 4)
  Q8_0: fp16 d = |N(0, 0.001)|, int8 quants uniform in -127..127                 (config 1)
  Q5_K: fp16 d, dmin = |N(0, 0.01)|, 6-bit sub-scales/mins and 5-bit quants uniform (config 2)
  Q6_K: fp16 d = |N(0, 0.01)|, int8 sub-scales uniform in -32..31, 6-bit quants uniform (config 2, 4 head)
  Q4_1: fp16 d = |N(0, 0.02)|, fp16 m = N(0, 0.02), 4-bit quants uniform
"""
from __future__ import annotations

import numpy as np

SEED = 0x5EED


def rng(config_id: int = 0, salt: int = 0) -> np.random.Generator:
    return np.random.default_rng([SEED, config_id, salt])


def _f16(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float16).view(np.uint8).reshape(a.shape + (2,))


def q4_0(r: np.random.Generator, rows: int, cols: int, d_sigma: float = 0.02) -> np.ndarray:
    nb = cols // 32
    d = _f16(np.abs(r.normal(0.0, d_sigma, (rows, nb))).astype(np.float32))
    qs = r.integers(0, 256, (rows, nb, 16), dtype=np.uint8)
    return np.concatenate([d, qs], axis=2).reshape(rows, nb * 18)


def q8_0(r: np.random.Generator, rows: int, cols: int, d_sigma: float = 0.001) -> np.ndarray:
    nb = cols // 32
    d = _f16(np.abs(r.normal(0.0, d_sigma, (rows, nb))).astype(np.float32))
    qs = r.integers(-127, 128, (rows, nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    return np.concatenate([d, qs], axis=2).reshape(rows, nb * 34)


def q4_1(r: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    nb = cols // 32
    d = _f16(np.abs(r.normal(0.0, 0.02, (rows, nb))).astype(np.float32))
    m = _f16(r.normal(0.0, 0.02, (rows, nb)).astype(np.float32))
    qs = r.integers(0, 256, (rows, nb, 16), dtype=np.uint8)
    return np.concatenate([d, m, qs], axis=2).reshape(rows, nb * 20)


def q5_k(r: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    nsb = cols // 256
    d = _f16(np.abs(r.normal(0.0, 0.01, (rows, nsb))).astype(np.float32))
    dmin = _f16(np.abs(r.normal(0.0, 0.01, (rows, nsb))).astype(np.float32))
    rest = r.integers(0, 256, (rows, nsb, 172), dtype=np.uint8)  # 12 packed scales, 32 qh, 128 qs
    return np.concatenate([d, dmin, rest], axis=2).reshape(rows, nsb * 176)


def q6_k(r: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    nsb = cols // 256
    q = r.integers(0, 256, (rows, nsb, 192), dtype=np.uint8)  # ql[128], qh[64]
    sc = r.integers(-32, 32, (rows, nsb, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
    d = _f16(np.abs(r.normal(0.0, 0.01, (rows, nsb))).astype(np.float32))
    return np.concatenate([q, sc, d], axis=2).reshape(rows, nsb * 210)


GEN = {2: q4_0, 8: q8_0, 3: q4_1, 13: q5_k, 14: q6_k}


def matrix(fmt: int, r: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    return GEN[fmt](r, rows, cols)


def activation(r: np.random.Generator, n: int, sigma: float = 1.0) -> np.ndarray:
    return r.normal(0.0, sigma, n).astype(np.float32)
