"""GEMM case statements in FP64.

The reference's case is ``C = A @ B`` with B [K, N] (knowledge/seed/cases/gemm_fp16.yaml:8-13),
executed in FP64 on the exact input bytes by src/kta/checks/scripts/ref_torch.py:28-38; the
B200 cases state ``C = A @ B.T`` with B [N, K]. Inputs here are float64 arrays already widened
exactly (oracle.numerics).
"""

from __future__ import annotations

import numpy as np


def gemm_tn(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """C = A @ B.T in float64; A [M, K], B [N, K]."""
    return np.asarray(a, dtype=np.float64) @ np.asarray(b, dtype=np.float64).T


def gemm_nn(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """C = A @ B in float64; A [M, K], B [K, N] (the reference's own case statement)."""
    return np.asarray(a, dtype=np.float64) @ np.asarray(b, dtype=np.float64)


def gemm_tn_rows(a: np.ndarray, b: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """Rows ``rows`` of A @ B.T only: full-size checks at a fraction of the FLOPs."""
    return np.asarray(a[rows], dtype=np.float64) @ np.asarray(b, dtype=np.float64).T


def moe_gemm(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """MoE expert GEMM in float64 (KTA's moe_gemm, perfmodel/testset/gen.py:332-356): A [T, K]
    with T / E consecutive rows per expert, W [E, K, N]; C[rows of e] = A[rows of e] @ W[e]."""
    e = w.shape[0]
    per = a.shape[0] // e
    a64, w64 = np.asarray(a, np.float64), np.asarray(w, np.float64)
    return np.concatenate([a64[i * per:(i + 1) * per] @ w64[i] for i in range(e)], axis=0)
