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


# Shapes the default routing sends to the 2-SM pair kernel (256x256 tiles over CTA pairs):
# pair tiles >= SMs / 2 and no more waves than 128x256 tiles on 148 SMs, e.g. 3000 x 2904:
# 12 x 12 = 144 pair tiles (2 waves of 74) against 24 x 12 = 288 one-SM tiles (2 waves of 148).
# Every one has ragged M and N (not multiples of 256) and most a K tail (not a multiple of 64).
PAIR_SHAPES = [
    (3000, 2904, 1000),
    (2304, 4352, 264),
    (4100, 2600, 1032),
    (2200, 2312, 72),
]


@pytest.mark.parametrize("route", ["default", "force"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", PAIR_SHAPES)
def test_gemm_pair_kernel_ragged(cuda_device, monkeypatch, m, n, k, dtype, route):
    """The 2-SM pair kernel on ragged edges, by the default routing and with
    KTA_GEMM_PAIR=force (read on every call)."""
    from kta_b200 import ops

    if route == "force":
        monkeypatch.setenv("KTA_GEMM_PAIR", "force")
    else:
        monkeypatch.delenv("KTA_GEMM_PAIR", raising=False)
    a, b = _inputs(m, n, k, dtype, seed=3)
    c = torch.full((m, n), float("nan"), dtype=dtype, device=cuda_device)
    ops.gemm(a.to(cuda_device), b.to(cuda_device), out=c)
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))


@pytest.mark.parametrize("route", ["default", "force", "off"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,n,k", PAIR_SHAPES)
def test_gemm_nn_pair_kernel_ragged(cuda_device, monkeypatch, m, n, k, dtype, route):
    """The reference's layout C = A @ B (B [K, N], an MN-major operand in 64-column blocks)
    through the 2-SM pair kernel on ragged edges, by the default routing, KTA_GEMM_PAIR=force
    and, for comparison, the one-SM kernel (KTA_GEMM_PAIR=0)."""
    from kta_b200 import ops

    if route == "default":
        monkeypatch.delenv("KTA_GEMM_PAIR", raising=False)
    else:
        monkeypatch.setenv("KTA_GEMM_PAIR", "force" if route == "force" else "0")
    a, b = _inputs(m, n, k, dtype, seed=5, b_layout="kn")
    c = torch.full((m, n), float("nan"), dtype=dtype, device=cuda_device)
    ops.gemm(a.to(cuda_device), b.to(cuda_device), out=c, b_layout="kn")
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_nn(a.double().numpy(), b.double().numpy()))


@pytest.mark.parametrize("route", ["force", "off"])
@pytest.mark.parametrize("m,n,k", [(520, 1000, 136), (129, 384, 64), (700, 904, 320)])
def test_gemm_small_shapes_on_both_kernels(cuda_device, monkeypatch, m, n, k, route):
    """Shapes the default routing keeps on the 1-SM kernel, forced onto the pair kernel
    (M > 128), and the pair kernel switched off."""
    from kta_b200 import ops

    monkeypatch.setenv("KTA_GEMM_PAIR", route if route == "force" else "0")
    a, b = _inputs(m, n, k, torch.bfloat16, seed=4)
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))


@pytest.mark.parametrize("route", ["default", "force", "off"])
def test_gemm_8192_with_k_tail_sampled_rows(cuda_device, monkeypatch, route):
    """8192 x 8192 x 8200: the headline shape with a K tail of 8 (not a multiple of the 64-deep
    stage) on the pair kernel (default and forced) and on the 1-SM kernel; 100 sampled rows
    against FP64."""
    from kta_b200 import ops

    if route == "default":
        monkeypatch.delenv("KTA_GEMM_PAIR", raising=False)
    else:
        monkeypatch.setenv("KTA_GEMM_PAIR", "force" if route == "force" else "0")
    m, n, k = 8192, 8192, 8200
    a, b = _inputs(m, n, k, torch.bfloat16, seed=6)
    c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    ops.gemm(a.to(cuda_device), b.to(cuda_device), out=c)
    torch.cuda.synchronize()
    rows = np.random.default_rng(2).choice(m, size=96, replace=False)
    rows = np.concatenate([rows, [0, 255, 256, m - 1]])
    ref = ogemm.gemm_tn_rows(a.double().numpy(), b.double().numpy(), rows)
    _check(c[torch.as_tensor(rows)], ref)
    assert not torch.isnan(c.float()).any()


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("m,n,k", [(1000, 1032, 264), (3000, 2904, 1000), (16, 4096, 1024),
                                   (40, 2048, 512)])
def test_gemm_padded_leading_dimensions(cuda_device, m, n, k, layout):
    """A, B and C as views into wider row-major buffers (lda, ldb, ldc larger than the logical
    row, all multiples of 8): every path reads and writes through the leading dimensions, and
    the padding columns of C stay untouched."""
    from kta_b200 import ops

    pad = 24
    a, b = _inputs(m, n, k, torch.bfloat16, seed=9, b_layout=layout)
    abuf = torch.zeros(m, k + pad, dtype=torch.bfloat16, device=cuda_device)
    abuf[:, :k] = a.to(cuda_device)
    rows_b, cols_b = b.shape
    bbuf = torch.zeros(rows_b, cols_b + pad, dtype=torch.bfloat16, device=cuda_device)
    bbuf[:, :cols_b] = b.to(cuda_device)
    cbuf = torch.full((m, n + pad), 7.0, dtype=torch.bfloat16, device=cuda_device)
    c = cbuf[:, :n]
    ops.gemm(abuf[:, :k], bbuf[:, :cols_b], out=c, b_layout=layout)
    torch.cuda.synchronize()
    ref = (ogemm.gemm_tn if layout == "nk" else ogemm.gemm_nn)(a.double().numpy(),
                                                               b.double().numpy())
    _check(c, ref)
    assert torch.all(cbuf[:, n:] == 7.0)


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


def test_gemm_host_returns_with_c_on_the_host(cuda_device):
    """With the default wait=True the result is complete on return: read at once, no sync."""
    from kta_b200 import ops

    a, b = _inputs(1536, 1024, 512, torch.bfloat16, seed=8)
    c = ops.gemm_host(a.pin_memory(), b.pin_memory())
    _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))


def test_gemm_host_two_streams_in_flight_with_different_inputs(cuda_device):
    """Four calls in flight at once, alternating between two caller streams, each with its own
    inputs and output (wait=False): each stream gets device buffers of its own and consecutive
    calls on one stream reuse them only after the previous read-back, so no call reads or
    returns another call's data."""
    from kta_b200 import ops

    m, n, k = 2048, 1536, 1024
    sets = [_inputs(m, n, k, torch.bfloat16, seed=20 + i) for i in range(4)]
    pinned = [(a.pin_memory(), b.pin_memory()) for a, b in sets]
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16).pin_memory()
            for _ in range(4)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for i in range(4):
        with torch.cuda.stream(streams[i % 2]):
            ops.gemm_host(*pinned[i], out=outs[i], wait=False)
    torch.cuda.synchronize()
    for (a, b), c in zip(sets, outs):
        _check(c, ogemm.gemm_tn(a.double().numpy(), b.double().numpy()))
