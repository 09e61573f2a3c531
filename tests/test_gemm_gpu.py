"""GEMM parity on the GPU: libkta_b200 (through the C ABI) against the FP64 oracle.

Inputs are seeded N(0,1)/sqrt(K) (the B200 cases' distribution), identical bytes go to the
kernel and to the oracle. Tolerance: |y - ref| <= atol + rtol*|ref| with rtol = atol = 1e-2
for bf16 and f16 outputs, as the cases' contracts state.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gemm as ogemm

RTOL = ATOL = 1e-2

pytestmark = pytest.mark.gpu


def _inputs(m: int, n: int, k: int, dtype: torch.dtype, seed: int = 0, b_layout: str = "nk"):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) / k**0.5).to(dtype)
    shape_b = (n, k) if b_layout == "nk" else (k, n)
    b = (torch.randn(*shape_b, generator=g) / k**0.5).to(dtype)
    return a, b


def _check(got: torch.Tensor, ref: np.ndarray) -> None:
    y = got.double().cpu().numpy()
    err = np.abs(y - ref)
    bad = err > ATOL + RTOL * np.abs(ref)
    assert np.isfinite(y).all(), "non-finite output (unwritten or NaN elements)"
    assert not bad.any(), f"{int(bad.sum())} mismatches, max err {err.max():.3e}"


SHAPES = [
    (128, 256, 64),
    (256, 512, 1024),
    (1024, 1024, 1024),
    (300, 520, 200),
    (129, 136, 72),
    (2048, 2048, 2048),
    (4096, 1024, 512),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_tn(cuda_device, m, n, k, dtype):
    from kta_b200 import ops

    a, b = _inputs(m, n, k, dtype)
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (1024, 1024, 1024), (300, 520, 200),
                                   (4096, 4096, 512)])
def test_gemm_nn_reference_layout(cuda_device, m, n, k, dtype):
    """The reference's own statement C = A @ B with B [K, N] row-major."""
    from kta_b200 import ops

    a, b = _inputs(m, n, k, dtype, b_layout="kn")
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device), b_layout="kn")
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_nn(a.double().numpy(), b.double().numpy()))


@pytest.mark.parametrize("m", [1, 16, 17, 33, 64])
@pytest.mark.parametrize("n,k", [(8192, 8192), (520, 200), (1024, 4096)])
def test_gemm_skinny(cuda_device, m, n, k):
    from kta_b200 import ops

    a, b = _inputs(m, n, k, torch.bfloat16)
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m", [1, 5, 16])
@pytest.mark.parametrize("n,k", [(1000, 200), (1184, 8200), (9472, 264), (16384, 512), (8, 16)])
def test_gemm_m16_every_sm_path(cuda_device, m, n, k, dtype):
    """M <= 16 runs on mma.sync with N cut into n8 tiles over one wave of CTAs: K tails
    (200, 264, 8200 are not multiples of the 256-deep stage), N = 8 (one tile), N = 9472 (8
    tiles on each of 148 SMs) and N = 16384 (more than one wave: the tensor-memory kernel)."""
    from kta_b200 import ops

    a, b = _inputs(m, n, k, dtype, seed=5)
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))


def test_gemm_bf16_8192_sampled_rows(cuda_device):
    """The full 8192^3 bf16 config; 96 sampled rows checked against FP64."""
    from kta_b200 import ops

    m = n = k = 8192
    a, b = _inputs(m, n, k, torch.bfloat16)
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    rows = np.random.default_rng(1).choice(m, size=96, replace=False)
    rows = np.concatenate([rows, [0, 127, 128, m - 1]])
    ref = ogemm.gemm_tn_rows(a.double().numpy(), b.double().numpy(), rows)
    _check(c[torch.as_tensor(rows)], ref)
    assert torch.isfinite(c.float()).all()


def test_gemm_is_deterministic(cuda_device):
    from kta_b200 import ops

    a, b = _inputs(1024, 2048, 4096, torch.bfloat16)
    a, b = a.to(cuda_device), b.to(cuda_device)
    c1 = ops.gemm(a, b)
    c2 = ops.gemm(a, b)
    torch.cuda.synchronize()
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))


def test_gemm_writes_every_element_of_a_nan_filled_output(cuda_device):
    """The reference's NaN-fill coverage check (src/kta/measure/bench.py:106-109)."""
    from kta_b200 import ops

    a, b = _inputs(700, 904, 320, torch.float16)
    c = torch.full((700, 904), float("nan"), dtype=torch.float16, device=cuda_device)
    ops.gemm(a.to(cuda_device), b.to(cuda_device), out=c)
    torch.cuda.synchronize()
    assert not torch.isnan(c).any()


def test_device_status_clean_after_gemms(cuda_device):
    from kta_b200 import lib

    assert lib.device_status(clear=True)[0] == 0


@pytest.mark.parametrize("m,n,k,chunks", [(1000, 520, 256, 3), (4096, 2048, 1024, 8),
                                          (100, 64, 64, 8)])
def test_gemm_host_buffers_pipelined(cuda_device, m, n, k, chunks):
    """The host-buffer entry: pinned A, B in, pinned C out, copies overlapped with the GEMM
    row blocks on three streams."""
    from kta_b200 import ops

    a, b = _inputs(m, n, k, torch.bfloat16)
    c = ops.gemm_host(a.pin_memory(), b.pin_memory(), chunks=chunks)
    torch.cuda.synchronize()
    assert not c.is_cuda
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))
