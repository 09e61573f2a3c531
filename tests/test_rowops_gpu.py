"""Row RMSNorm and softmax on the GPU through the C ABI against the FP64 oracle
(oracle/rowops.py, pinned to the reference's statement runner). f16 and bf16; every
threads-per-row configuration of the launcher (N = 8 ... 16384), ragged row counts, the
reference's test-set shapes (gen.py:249-252), large magnitudes for the softmax's max
subtraction, NaN-filled outputs fully written, repeat runs byte-identical, and the
reference-compatible `so` shims. Tolerance: |y - ref| <= atol + rtol |ref| with rtol 1e-2,
atol 1e-2 (RMSNorm) / 1e-3 (softmax, whose outputs are below 1)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import rowops as orow

pytestmark = pytest.mark.gpu

SHAPES = [(1, 8), (3, 40), (5, 264), (33, 512), (2048, 1024), (1024, 2048), (512, 4096),
          (768, 3072), (77, 8192), (7, 12288), (5, 16384)]
DTYPES = [torch.float16, torch.bfloat16]


def _x(m, n, dtype, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(m, n, generator=g) * scale).to(dtype)


def _check(y, ref, atol):
    got = y.double().cpu().numpy()
    err = np.abs(got - ref)
    bad = err > atol + 1e-2 * np.abs(ref)
    assert np.isfinite(got).all()
    assert not bad.any(), f"{int(bad.sum())} mismatches, max err {err.max():.3e}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n", SHAPES)
def test_rmsnorm(cuda_device, m, n, dtype):
    from kta_b200 import ops

    x = _x(m, n, dtype)
    w = _x(1, n, dtype, seed=1).reshape(n)
    y = ops.rmsnorm(x.to(cuda_device), w.to(cuda_device), 1e-6)
    torch.cuda.synchronize()
    _check(y, orow.rmsnorm(x.double().numpy(), w.double().numpy(), 1e-6), 1e-2)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("m,n", SHAPES)
def test_softmax(cuda_device, m, n, dtype):
    from kta_b200 import ops

    x = _x(m, n, dtype, scale=3.0)
    y = ops.softmax(x.to(cuda_device))
    torch.cuda.synchronize()
    _check(y, orow.softmax(x.double().numpy()), 1e-3)
    assert torch.allclose(y.float().sum(-1).cpu(), torch.ones(m), atol=2e-2)


def test_softmax_large_magnitudes_and_constant_rows(cuda_device):
    from kta_b200 import ops

    x = _x(64, 2048, torch.float16, scale=1.0)
    x[:16] *= 3000.0                      # |x| up to ~1e4: exp needs the max subtracted
    x[16:32] = 7.0                        # constant rows: uniform 1/N
    x[32:48, 5] = 60000.0                 # one dominant entry per row
    y = ops.softmax(x.to(cuda_device))
    torch.cuda.synchronize()
    _check(y, orow.softmax(x.double().numpy()), 1e-3)


def test_rmsnorm_zero_rows_and_eps(cuda_device):
    from kta_b200 import ops

    x = _x(16, 1024, torch.float16)
    x[3] = 0.0
    w = torch.ones(1024, dtype=torch.float16)
    for eps in (1e-6, 1e-2):
        y = ops.rmsnorm(x.to(cuda_device), w.to(cuda_device), eps)
        torch.cuda.synchronize()
        _check(y, orow.rmsnorm(x.double().numpy(), w.double().numpy(), eps), 1e-2)
        assert torch.count_nonzero(y[3]).item() == 0


@pytest.mark.parametrize("op", ["rmsnorm", "softmax"])
def test_nan_fill_coverage_and_determinism(cuda_device, op):
    from kta_b200 import ops

    x = _x(1000, 4096, torch.bfloat16).to(cuda_device)
    w = _x(1, 4096, torch.bfloat16, seed=3).reshape(4096).to(cuda_device)
    run = (lambda out: ops.rmsnorm(x, w, 1e-6, out=out)) if op == "rmsnorm" else \
        (lambda out: ops.softmax(x, out=out))
    y1 = torch.full_like(x, float("nan"))
    run(y1)
    y2 = run(None)
    torch.cuda.synchronize()
    assert not torch.isnan(y1).any()
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))


def test_so_shims_match_the_entries(cuda_device):
    from kta_b200 import lib, ops

    L = lib.load()
    x = _x(256, 1024, torch.float16).to(cuda_device)
    w = _x(1, 1024, torch.float16, seed=2).reshape(1024).to(cuda_device)
    y = torch.empty_like(x)
    L.kta_so_rmsnorm_f16(x.data_ptr(), w.data_ptr(), y.data_ptr(), 256, 1024)
    torch.cuda.synchronize()
    assert L.kta_last_error() == 0
    assert torch.equal(y, ops.rmsnorm(x, w, 1e-6))
    L.kta_so_softmax_f16(x.data_ptr(), y.data_ptr(), 256, 1024)
    torch.cuda.synchronize()
    assert L.kta_last_error() == 0
    assert torch.equal(y, ops.softmax(x))


@pytest.mark.parametrize("case", ["rmsnorm_f16", "softmax_f16"])
def test_quick_check_of_the_cases(cuda_device, case):
    from kta_b200 import checkflow, schemas

    res = checkflow.quick_check(schemas.load_case_file(case))
    assert res["passed"], res["failures"]
