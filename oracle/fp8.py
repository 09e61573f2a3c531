"""Block-scaled FP8 statement in float64, and the e4m3 block quantiser of its inputs.

The B200 FP8 case (kta_b200/cases/gemm_fp8_blockscaled.yaml) dequantises e4m3 codes with
fp32 scales per 1x128 activation block and per 128x128 weight block and multiplies in FP64;
the reference's TileLang fp8gemm (perfmodel/testset/gen.py:306-329) is the same contraction
C = A B^T without scales. Codes are decoded exactly (oracle.numerics).
"""

from __future__ import annotations

import numpy as np

from oracle import numerics

BLOCK = 128


def dequant_rows(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Activation A [M, K]: value = e4m3(code) * sa[m, k // 128]."""
    x = numerics.e4m3_bits_to_f64(codes)
    k = x.shape[1]
    return x * np.repeat(scales.astype(np.float64), BLOCK, axis=1)[:, :k]


def dequant_blocks(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Weight B [N, K]: value = e4m3(code) * sb[n // 128, k // 128]."""
    x = numerics.e4m3_bits_to_f64(codes)
    n, k = x.shape
    s = np.repeat(np.repeat(scales.astype(np.float64), BLOCK, axis=0), BLOCK, axis=1)
    return x * s[:n, :k]


def gemm_blockscaled(a_codes, sa, b_codes, sb) -> np.ndarray:
    """C = dequant(A) @ dequant(B).T in float64."""
    return dequant_rows(a_codes, sa) @ dequant_blocks(b_codes, sb).T


def quantize(x: np.ndarray, block_rows: int) -> tuple[np.ndarray, np.ndarray]:
    """e4m3 codes and fp32 scales amax/448 per (block_rows x 128) block, round to nearest
    even, the quantiser the case's inputs go through (numpy restatement)."""
    x = np.asarray(x, dtype=np.float32)
    rows, cols = x.shape
    rb, cb = -(-rows // block_rows), -(-cols // BLOCK)
    pad = np.zeros((rb * block_rows, cb * BLOCK), dtype=np.float32)
    pad[:rows, :cols] = x
    blocks = pad.reshape(rb, block_rows, cb, BLOCK)
    amax = np.abs(blocks).max(axis=(1, 3))
    scale = np.where(amax > 0, amax / np.float32(numerics.E4M3_MAX), np.float32(1.0))
    scale = scale.astype(np.float32)
    q = (blocks / scale[:, None, :, None]).astype(np.float32)
    q = q.reshape(rb * block_rows, cb * BLOCK)[:rows, :cols]
    return numerics.f64_to_e4m3_bits(q.astype(np.float64)), scale
