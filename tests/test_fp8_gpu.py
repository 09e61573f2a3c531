"""FP8 block-scaled GEMM parity on the GPU: kta_gemm_fp8_blockscaled through the C ABI
against the FP64 product of the dequantised inputs (the case statement). Source values
N(0,1) with 1% outliers x20, quantised to e4m3 with fp32 scales amax/448 per 1x128
(activations) and 128x128 (weights). Tolerance: |y - ref| <= 2e-2 |ref| + 2e-2, and the
relative L2 error below 2e-2."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8

pytestmark = pytest.mark.gpu


def _make(m, n, k, seed=0):
    g = np.random.default_rng(seed)
    a = g.standard_normal((m, k)) * np.where(g.random((m, k)) < 0.01, 20.0, 1.0)
    b = g.standard_normal((n, k)) * np.where(g.random((n, k)) < 0.01, 20.0, 1.0)
    ac, sa = ofp8.quantize(a, 1)
    bc, sb = ofp8.quantize(b, 128)
    return ac, sa, bc, sb


def _run(dev, ac, sa, bc, sb):
    from kta_b200 import ops

    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
    c = ops.gemm_fp8_blockscaled(t(ac).view(torch.float8_e4m3fn), t(sa),
                                 t(bc).view(torch.float8_e4m3fn), t(sb))
    torch.cuda.synchronize()
    return c.double().cpu().numpy()


def _check(y, ref):
    assert np.isfinite(y).all()
    err = np.abs(y - ref)
    bad = err > 2e-2 * np.abs(ref) + 2e-2
    assert not bad.any(), f"{int(bad.sum())} mismatches, max err {err.max():.3e}"
    assert np.linalg.norm(y - ref) <= 2e-2 * np.linalg.norm(ref)


# 18944 x 256: 148 tiles of 128 x 256, exactly one per SM of a B200. 19072 x 256: 149 tiles,
# the last cut into four 128 x 64 quarters; 19200 x 264: 300 tiles, the 4 of the last round
# cut into quarters, three of each lying wholly past N = 264 (they write nothing).
@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (256, 512, 1024), (300, 520, 208),
                                   (1, 256, 128), (130, 136, 4096), (512, 1024, 7168),
                                   (18944, 256, 256), (19072, 256, 256), (19200, 264, 384)])
def test_fp8_blockscaled(cuda_device, m, n, k):
    ac, sa, bc, sb = _make(m, n, k)
    y = _run(cuda_device, ac, sa, bc, sb)
    _check(y, ofp8.gemm_blockscaled(ac, sa, bc, sb))


def test_fp8_blockscaled_baseline_config_sampled_rows(cuda_device):
    """M=4096, N=7168, K=7168: 64 sampled rows checked against FP64."""
    m, n, k = 4096, 7168, 7168
    ac, sa, bc, sb = _make(m, n, k, seed=1)
    y = _run(cuda_device, ac, sa, bc, sb)
    # rows 3072 .. 4095 hold the 8 tiles of the last round (cut into quarters), columns
    # 6912 .. 7167
    rows = np.concatenate([np.random.default_rng(2).choice(m, 60, replace=False),
                           [0, 127, 128, 3072, 3500, 3583, 3584, m - 1]])
    ref = ofp8.dequant_rows(ac[rows], sa[rows]) @ ofp8.dequant_blocks(bc, sb).T
    _check(y[rows], ref)


def test_fp8_quarters_match_whole_tiles(cuda_device, monkeypatch):
    """The tail quarters give the same bits as the same tiles computed whole
    (KTA_FP8_SPLIT=0): the same products and the same fp32 promotion order."""
    ac, sa, bc, sb = _make(19072, 512, 512, seed=4)
    y1 = _run(cuda_device, ac, sa, bc, sb)
    monkeypatch.setenv("KTA_FP8_SPLIT", "0")
    y2 = _run(cuda_device, ac, sa, bc, sb)
    np.testing.assert_array_equal(y1, y2)


def test_fp8_uses_the_scales(cuda_device):
    """Doubling one weight block's scale doubles exactly that block's contribution."""
    ac, sa, bc, sb = _make(128, 256, 256, seed=3)
    y1 = _run(cuda_device, ac, sa, bc, sb)
    sb2 = sb.copy()
    sb2[1, 0] *= 2.0
    y2 = _run(cuda_device, ac, sa, bc, sb2)
    ref2 = ofp8.gemm_blockscaled(ac, sa, bc, sb2)
    _check(y2, ref2)
    assert np.allclose(y1[:, :128], y2[:, :128])
