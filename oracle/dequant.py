"""4-bit weight dequantisation and the dequantising GEMMs in float64 (numpy), test
infrastructure only.

B[n, k] = decode(code[n, k]) * Sc[n, k // G], codes two per byte (the lower nibble is the even
k), as KTA's test-set kernels define it:
- int4 (w4gemm, perfmodel/testset/gen.py:359-414, :389-397): decode(x) = x - 8 (x in 0..15);
- e2m1 (nvfp4gemm, perfmodel/testset/gen.py:744-778, :766-771): e = (x >> 1) & 3, m = x & 1,
  magnitude (2 + m) << (e - 1) for e > 0 else m, times 0.5, negative when x >= 8.
The reference computes the product in f16: here decode * scale is formed exactly (at most 15
significant bits) and rounded once to f16, the same value. C = A @ B^T then in float64.
"""

from __future__ import annotations

import numpy as np


def unpack(bq: np.ndarray) -> np.ndarray:
    b = np.asarray(bq).view(np.uint8).astype(np.int64)
    n, half = b.shape
    out = np.empty((n, 2 * half), dtype=np.int64)
    out[:, 0::2] = b & 15
    out[:, 1::2] = b >> 4
    return out


def decode(codes: np.ndarray, fmt: str) -> np.ndarray:
    if fmt == "int4":
        return (codes - 8).astype(np.float64)
    e, m = (codes >> 1) & 3, codes & 1
    mag = np.where(e > 0, (2 + m) << np.maximum(e - 1, 0), m).astype(np.float64) * 0.5
    return np.where(codes >= 8, -mag, mag)


def dequant(bq: np.ndarray, sc: np.ndarray, fmt: str, group: int) -> np.ndarray:
    codes = unpack(bq)
    s = np.repeat(np.asarray(sc, dtype=np.float16).astype(np.float64), group, axis=1)
    exact = decode(codes, fmt) * s[:, :codes.shape[1]]
    return exact.astype(np.float16).astype(np.float64)


def gemm(a: np.ndarray, bq: np.ndarray, sc: np.ndarray, fmt: str, group: int) -> np.ndarray:
    return np.asarray(a, dtype=np.float64) @ dequant(bq, sc, fmt, group).T
