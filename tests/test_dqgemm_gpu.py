"""GEMM with a 4-bit B dequantised in the main loop (w4a16 int4 and NVFP4 e2m1) on the GPU
through the C ABI against the FP64 oracle (oracle/dequant.py: B rounded to f16 as the
reference's kernel computes it, then FP64 A @ B^T; pinned to the reference's statement runner).
Group sizes 16-128, ragged M and N, K tails of whole stages, the test set's 2048^3 shape,
NaN-filled output fully written, and the `so` shims. Tolerance |y - ref| <= 1e-2 + 1e-2 |ref|
with A ~ N(0,1)/sqrt(K)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import dequant

pytestmark = pytest.mark.gpu


def _inputs(m, n, k, fmt, group, seed=0):
    from kta_b200.inputs import quantize_4bit

    g = np.random.default_rng(seed)
    a = (g.standard_normal((m, k)) / np.sqrt(k)).astype(np.float16)
    src = g.standard_normal((n, k)).astype(np.float32)
    bq, sc = quantize_4bit(src, fmt, group)
    return a, bq, sc


def _run(dev, a, bq, sc, fmt, group):
    from kta_b200 import ops

    c = ops.gemm_4bit(torch.from_numpy(a).to(dev), torch.from_numpy(bq).to(dev),
                      torch.from_numpy(sc).to(dev), fmt, group)
    torch.cuda.synchronize()
    return c.double().cpu().numpy()


def _check(y, ref):
    err = np.abs(y - ref)
    assert np.isfinite(y).all()
    bad = err > 1e-2 + 1e-2 * np.abs(ref)
    assert not bad.any(), f"{int(bad.sum())} mismatches, max err {err.max():.3e}"


@pytest.mark.parametrize("group", [16, 32, 64, 128])
@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (300, 520, 256), (1, 64, 1024),
                                   (257, 136, 2048)])
def test_w4a16(cuda_device, m, n, k, group):
    a, bq, sc = _inputs(m, n, k, "int4", group)
    _check(_run(cuda_device, a, bq, sc, "int4", group), dequant.gemm(a, bq, sc, "int4", group))


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (300, 520, 256), (1, 64, 1024),
                                   (257, 136, 2048)])
def test_nvfp4(cuda_device, m, n, k):
    a, bq, sc = _inputs(m, n, k, "e2m1", 16, seed=1)
    _check(_run(cuda_device, a, bq, sc, "e2m1", 16), dequant.gemm(a, bq, sc, "e2m1", 16))


@pytest.mark.parametrize("fmt,group", [("int4", 32), ("e2m1", 16)])
def test_test_set_shape_sampled_rows(cuda_device, fmt, group):
    a, bq, sc = _inputs(2048, 2048, 2048, fmt, group, seed=2)
    y = _run(cuda_device, a, bq, sc, fmt, group)
    rows = np.r_[0:8, 1000:1008, 2040:2048]
    ref = a[rows].astype(np.float64) @ dequant.dequant(bq, sc, fmt, group).T
    _check(y[rows], ref)


@pytest.mark.parametrize("reps", [1, 5])
@pytest.mark.parametrize("scale", [0.25, 2.0 ** -20])
def test_every_code_and_nibble_order(cuda_device, scale, reps):
    """All 16 codes in both nibble positions, with power-of-two scales (exact products; 2^-20
    is an f16 subnormal, so the decoded values are subnormal too). A is the identity stacked
    `reps` times: M = 64 runs the single-CTA kernel, M = 320 the CTA-pair kernel."""
    n, k = 128, 64
    codes = np.tile(np.arange(16, dtype=np.uint8), (n, k // 16))
    codes = np.roll(codes, 3, axis=1)
    bq = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8).view(np.int8)
    for fmt, group in (("int4", 32), ("e2m1", 16)):
        sc = np.full((n, k // group), scale, dtype=np.float16)
        eye = np.tile(np.eye(k, dtype=np.float16), (reps, 1))
        y = _run(cuda_device, np.ascontiguousarray(eye), bq, sc, fmt, group)
        np.testing.assert_array_equal(y, np.tile(dequant.dequant(bq, sc, fmt, group).T,
                                                 (reps, 1)))


def test_nan_fill_and_so_shims(cuda_device):
    from kta_b200 import lib, ops

    L = lib.load()
    for fmt, group, shim in (("int4", 32, "kta_so_w4gemm_f16"),
                             ("e2m1", 16, "kta_so_nvfp4gemm_f16")):
        a, bq, sc = (torch.from_numpy(x).to(cuda_device)
                     for x in _inputs(512, 256, 512, fmt, group, seed=3))
        c1 = torch.full((512, 256), float("nan"), dtype=torch.float16, device=cuda_device)
        ops.gemm_4bit(a, bq, sc, fmt, group, out=c1)
        c2 = torch.full_like(c1, float("nan"))
        getattr(L, shim)(a.data_ptr(), bq.data_ptr(), sc.data_ptr(), c2.data_ptr(), 512, 256, 512)
        torch.cuda.synchronize()
        assert L.kta_last_error() == 0
        assert not torch.isnan(c1).any()
        assert torch.equal(c1, c2)


@pytest.mark.parametrize("case", ["w4gemm_f16", "nvfp4gemm_f16"])
def test_quick_check_of_the_cases(cuda_device, case):
    from kta_b200 import checkflow, schemas

    res = checkflow.quick_check(schemas.load_case_file(case))
    assert res["passed"], res["failures"]
