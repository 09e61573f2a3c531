"""Row-operation restatements in float64 (numpy), test infrastructure only.

- ``rmsnorm``: Y = X * rsqrt(mean_j X^2 + eps) * W per row, the function of KTA's test-set
  rmsnorm (perfmodel/testset/gen.py:662-704: fp32 sum of squares, rsqrt(ss / N + 1e-6),
  multiplied by W);
- ``softmax``: softmax per row, the function of the test-set softmax
  (perfmodel/testset/gen.py:781-807: exp2 of x log2(e) minus the row maximum, divided by the
  row sum; exp2(x log2 e) = exp(x)).
"""

from __future__ import annotations

import numpy as np


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(ms + eps) * np.asarray(w, dtype=np.float64)


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    e = np.exp(x - np.max(x, axis=-1, keepdims=True))
    return e / np.sum(e, axis=-1, keepdims=True)
