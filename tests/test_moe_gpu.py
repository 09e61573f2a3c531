"""MoE expert GEMM on the GPU through the C ABI against the FP64 oracle (oracle/gemm.py
moe_gemm, pinned to the reference's statement runner): f16 and bf16, one to eight experts,
K tails, the reference's test-set shape (E=8 T=2048 N=1024 K=2048), NaN-filled output fully
written, and the `so` shim. Tolerance |y - ref| <= 1e-2 + 1e-2 |ref| (inputs N(0,1)/sqrt(K))."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gemm as ogemm

pytestmark = pytest.mark.gpu


def _inputs(e, t, n, k, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(t, k, generator=g) / k ** 0.5).to(dtype)
    w = (torch.randn(e, k, n, generator=g) / k ** 0.5).to(dtype)
    return a, w


def _check(c, ref):
    y = c.double().cpu().numpy()
    err = np.abs(y - ref)
    assert np.isfinite(y).all()
    bad = err > 1e-2 + 1e-2 * np.abs(ref)
    assert not bad.any(), f"{int(bad.sum())} mismatches, max err {err.max():.3e}"


# Routes: "default" (2-SM 256 x 128 pair tiles when every expert's rows are a multiple of 256
# and the pair grid takes no more waves, else 128-row tiles on single SMs), "0"
# (KTA_GEMM_PAIR=0: single SMs), "force" (pairs whenever the rows allow). Experts of 512 and
# 256 rows with ragged N (520, 264) and K tails (200, 72) reach the pair kernel.
@pytest.mark.parametrize("route", ["default", "0", "force"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("e,t,n,k", [(1, 128, 64, 64), (2, 256, 256, 128), (4, 512, 520, 200),
                                     (3, 384, 1024, 1000), (8, 2048, 1024, 2048),
                                     (8, 1024, 768, 4096), (2, 1024, 520, 200),
                                     (4, 1024, 264, 72)])
def test_moe_gemm(cuda_device, monkeypatch, e, t, n, k, dtype, route):
    from kta_b200 import ops

    if route == "default":
        monkeypatch.delenv("KTA_GEMM_PAIR", raising=False)
    else:
        monkeypatch.setenv("KTA_GEMM_PAIR", route)
    a, w = _inputs(e, t, n, k, dtype)
    c = ops.moe_gemm(a.to(cuda_device), w.to(cuda_device))
    torch.cuda.synchronize()
    _check(c, ogemm.moe_gemm(a.double().numpy(), w.double().numpy()))


def test_moe_experts_are_not_mixed(cuda_device):
    """Expert e's rows see only W[e]: zero every expert but one."""
    from kta_b200 import ops

    a, w = _inputs(4, 512, 256, 256, torch.float16, seed=3)
    w[[0, 1, 3]] = 0
    c = ops.moe_gemm(a.to(cuda_device), w.to(cuda_device)).cpu()
    assert torch.count_nonzero(c[:256]) == 0 and torch.count_nonzero(c[384:]) == 0
    assert torch.count_nonzero(c[256:384]) > 0


def test_moe_experts_are_not_mixed_pair_tiles(cuda_device, monkeypatch):
    """The same with 256-row experts, on the 2-SM pair kernel: a pair tile's 256 rows and both
    CTAs' halves of W belong to one expert."""
    from kta_b200 import ops

    monkeypatch.setenv("KTA_GEMM_PAIR", "force")
    a, w = _inputs(4, 1024, 384, 256, torch.bfloat16, seed=4)
    w[[0, 1, 3]] = 0
    c = ops.moe_gemm(a.to(cuda_device), w.to(cuda_device)).cpu()
    assert torch.count_nonzero(c[:512]) == 0 and torch.count_nonzero(c[768:]) == 0
    assert torch.count_nonzero(c[512:768]) > 0
    ref = ogemm.moe_gemm(a.double().numpy(), w.double().numpy())
    _check(c, ref)


def test_moe_nan_fill_and_so_shim(cuda_device):
    from kta_b200 import lib, ops

    a, w = (x.to(cuda_device) for x in _inputs(8, 1024, 512, 512, torch.float16, seed=4))
    c1 = torch.full((1024, 512), float("nan"), dtype=torch.float16, device=cuda_device)
    ops.moe_gemm(a, w, out=c1)
    c2 = torch.full_like(c1, float("nan"))
    L = lib.load()
    L.kta_so_moe_gemm_f16(a.data_ptr(), w.data_ptr(), c2.data_ptr(), 8, 1024, 512, 512)
    torch.cuda.synchronize()
    assert L.kta_last_error() == 0
    assert not torch.isnan(c1).any()
    assert torch.equal(c1, c2)


def test_moe_quick_check_of_the_case(cuda_device):
    from kta_b200 import checkflow, schemas

    res = checkflow.quick_check(schemas.load_case_file("moe_gemm_f16"))
    assert res["passed"], res["failures"]
