"""The checker rejects what it must: quick checks of plug-in runners with a planted fault
(tests/planted_runners.py), as src/kta/checks/selftest.py:35-59 proves the reference's checker
on a missing row, an out-of-bounds store and a cuBLAS-linked module. Each planted mistake is
made on the host or by a correct kernel, so no GPU fault is involved. The correct entry on the
same case passes (the control)."""

from __future__ import annotations

import pytest

from kta_b200 import checkflow, schemas

pytestmark = pytest.mark.gpu

GEMM_SHAPE = {"M": 256, "N": 384, "K": 512}
PLANTED = "tests.planted_runners:"


def _failed(res, check):
    return [f for f in res["failures"] if f.get("check") == check]


def test_control_correct_entry_passes(cuda_device):
    cf = schemas.load_case_file("gemm_f16_1024")
    res = checkflow.quick_check(cf, GEMM_SHAPE)
    assert res["passed"], res["failures"]


def test_dropped_row_fails_numeric(cuda_device):
    cf = schemas.load_case_file("gemm_f16_1024")
    res = checkflow.quick_check(cf, GEMM_SHAPE, entry=PLANTED + "gemm_row_dropped")
    assert not res["passed"]
    bad = _failed(res, "numeric")
    assert bad and all("error" not in f for f in bad), res["failures"]
    # the unwritten row shows as non-finite elements: the NaN-fill coverage check
    assert any(f.get("nonfinite_where_ref_finite", 0) >= GEMM_SHAPE["N"] for f in bad), bad
    assert res["sub_checks"].get("anticheat") is True, res["failures"]  # library kernels only


def test_wrong_fp8_weight_scale_fails_numeric(cuda_device):
    cf = schemas.load_case_file("gemm_fp8_blockscaled")
    res = checkflow.quick_check(cf, GEMM_SHAPE, entry=PLANTED + "fp8_scale_doubled")
    assert not res["passed"]
    assert res["sub_checks"].get("anticheat") is True, res["failures"]
    bad = _failed(res, "numeric")
    assert bad and all("error" not in f for f in bad), res["failures"]


def test_foreign_kernel_fails_anticheat(cuda_device):
    cf = schemas.load_case_file("gemm_f16_1024")
    res = checkflow.quick_check(cf, GEMM_SHAPE, entry=PLANTED + "gemm_with_foreign_kernel")
    assert not res["passed"]
    bad = _failed(res, "anticheat.kernels")
    assert bad and all("undeclared kernel" in f.get("detail", "") for f in bad), res["failures"]
    assert res["sub_checks"].get("numeric") is True, res["failures"]  # the numbers are right


def test_nondeterministic_runner_fails_anticheat(cuda_device):
    cf = schemas.load_case_file("gemm_f16_1024")
    res = checkflow.quick_check(cf, GEMM_SHAPE, entry=PLANTED + "gemm_not_deterministic")
    assert not res["passed"]
    assert _failed(res, "anticheat.determinism"), res["failures"]
