"""Exact widening of 16- and 8-bit floating-point bit patterns to float64 (numpy only).

The reference widens inputs with ``arr.astype(np.float64)`` before running its statement
(src/kta/checks/scripts/ref_torch.py:32); numpy has no bf16 or e4m3 dtype, so the bit
patterns are decoded here from their definitions (IEEE-754 binary16; bfloat16 = the upper
half of binary32; OCP FP8 E4M3 "fn": bias 7, no infinities, S.1111.111 = NaN).
"""

from __future__ import annotations

import numpy as np


def bf16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    """uint16/int16 bf16 patterns -> float64 (exact)."""
    u = np.asarray(bits).view(np.uint16).astype(np.uint32) << 16
    return u.view(np.float32).astype(np.float64)


def f64_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float64 -> bf16 patterns (uint16), round to nearest even through float32.

    Double rounding (f64 -> f32 -> bf16) can differ from direct rounding only on exact
    ties of the f32 value, which the tests never rely on."""
    f = np.asarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    nan = np.isnan(f)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), out)


def f16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits).view(np.float16).astype(np.float64)


def _e4m3_table() -> np.ndarray:
    t = np.empty(256, dtype=np.float64)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_TABLE = _e4m3_table()
E4M3_MAX = 448.0


def e4m3_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(bits).view(np.uint8)]


def f64_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """Round to nearest even onto the e4m3 grid, saturating at +-448 (finite inputs)."""
    x = np.asarray(x, dtype=np.float64)
    finite = E4M3_TABLE[:0x7F]  # non-negative codes 0x00..0x7E, increasing
    a = np.minimum(np.abs(x), E4M3_MAX)
    idx = np.searchsorted(finite, a, side="left")
    idx = np.clip(idx, 1, len(finite) - 1)
    lo, hi = finite[idx - 1], finite[idx]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & ((idx & 1) == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(a == 0, 0, code).astype(np.uint8)
    sign = np.where(np.signbit(x), np.uint8(0x80), np.uint8(0))
    return (code | sign).astype(np.uint8)
