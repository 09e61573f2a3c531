"""The attention kernel's exp2 on the FMA pipe (kta_b200/csrc/attn.cu, exp2_poly_pair),
restated in numpy fp32 with the constants read from the source: Cody-Waite reduction by the
1.5 * 2^23 shifter, a degree-3 polynomial for 2^f on [-1/2, 1/2], 2^j added into the
exponent field. Its relative error must stay below 8e-5 (bf16 rounding of P is 3.9e-3) over
the inputs the kernel gives it (x <= 8, the rescale threshold), and every result must be a
positive normal number (the clamp at -125)."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parent.parent / "kta_b200" / "csrc" / "attn.cu"


def _coefficients() -> list[np.float32]:
    body = SRC.read_text()
    body = body[body.index("void exp2_poly_pair"):]
    body = body[:body.index("\n}\n")]
    lits = [float(x) for x in re.findall(r"f2\(([0-9.]+)f, \1f\)", body)]
    # shifter, then p = fma(c3, f, c2); p = fma(p, f, c1); p = fma(p, f, c0)
    assert len(lits) == 5 and lits[0] == 12582912.0
    c3, c2, c1, c0 = lits[1:]
    return [np.float32(c) for c in (c0, c1, c2, c3)]


def _fma32(a, b, c):
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x: np.ndarray) -> np.ndarray:
    c0, c1, c2, c3 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    shifter = np.float32(12582912.0)
    t = (x + shifter).astype(np.float32)
    f = (x - (t - shifter).astype(np.float32)).astype(np.float32)
    p = _fma32(np.full_like(f, c3), f, np.full_like(f, c2))
    p = _fma32(p, f, np.full_like(f, c1))
    p = _fma32(p, f, np.full_like(f, c0))
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def test_relative_error_bound():
    x = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
                        np.array([-0.5, 0.5, 0.0, -1e-7, 7.999], dtype=np.float32)])
    y = exp2_poly(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() < 8e-5, rel.max()


def test_clamp_gives_positive_normal_numbers():
    x = np.array([-np.inf, -1e30, -1000.0, -126.0, -125.6, -125.0], dtype=np.float32)
    y = exp2_poly(x)
    assert np.all(y > 0) and np.all(np.isfinite(y))
    assert np.all(y >= np.finfo(np.float32).tiny)
    assert np.all(y < 2.0 ** -124)


def test_polynomial_is_a_minimax_fit_not_a_taylor_series():
    c0, c1, c2, c3 = _coefficients()
    # a Taylor series would have c0 = 1 and c1 = ln 2 exactly; the fit trades them for a
    # smaller maximum error over the interval
    assert c0 != np.float32(1.0) and abs(float(c1) - np.log(2.0)) > 1e-6
