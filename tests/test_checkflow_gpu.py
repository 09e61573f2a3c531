"""The quick gate and the full check through libkta_b200 on the GPU: numeric on the
contract's distributions against the FP64 reference, the anti-cheat checks (only this
library's kernels launched, byte-identical repeat, no forbidden libraries linked)."""

from __future__ import annotations

import pytest

from kta_b200 import checkflow, schemas

pytestmark = pytest.mark.gpu


def test_quick_check_gemm_f16(cuda_device):
    cf = schemas.load_case_file("gemm_f16_1024")
    res = checkflow.quick_check(cf)
    assert res["passed"], res["failures"]
    assert res["sub_checks"] == {"numeric": True, "anticheat": True}


def test_full_check_attention_small_shape(cuda_device):
    cf = schemas.load_case_file("attn_causal")
    res = checkflow.full_check(cf, {"B": 1, "H": 2, "S": 384, "D": 128},
                               hidden_seed="0" * 32)
    assert res["passed"], res["failures"]
    assert res["detail"]["dists"] == cf.contract.input_dists
    # static scope: the hidden shapes are listed, not run
    assert res["detail"]["out_of_scope"] == list(checkflow.HIDDEN_CATEGORIES)


def test_anticheat_sees_only_library_kernels(cuda_device):
    cf = schemas.load_case_file("decode_gqa")
    shape = checkflow.case_shapes(cf)[0]
    small = {**shape, "B": 3, "max_seqlen": 300}
    res = checkflow.quick_check(cf, small)
    assert res["passed"], res["failures"]


# Every case of the library through the full check at a small shape of its own kind: numeric
# on every distribution of its contract, the anti-cheat checks, and the edge shapes; hidden
# shapes are listed as out of the static scope.
SMALL = {
    "attn_causal": {"B": 1, "H": 2, "S": 256, "D": 128},
    "decode_gqa": {"B": 3, "Hq": 32, "Hkv": 8, "D": 128, "max_seqlen": 300},
    "gemm_bf16_8192": {"M": 256, "N": 384, "K": 512},
    "gemm_f16_1024": {"M": 256, "N": 384, "K": 512},
    "gemm_f16_nn_ref": {"M": 256, "N": 384, "K": 512},
    "gemm_fp8_blockscaled": {"M": 256, "N": 384, "K": 512},
    "moe_gemm_f16": {"E": 2, "T": 256, "N": 256, "K": 256},
    "nvfp4gemm_f16": {"M": 256, "N": 256, "K": 256},
    "w4gemm_f16": {"M": 256, "N": 256, "K": 256},
    "rmsnorm_f16": {"M": 64, "N": 1024},
    "softmax_f16": {"M": 64, "N": 2048},
}


def test_small_shapes_cover_every_case():
    assert set(SMALL) == set(schemas.case_names())


@pytest.mark.parametrize("case", sorted(SMALL))
def test_full_check_every_case(cuda_device, case):
    cf = schemas.load_case_file(case)
    res = checkflow.full_check(cf, SMALL[case], hidden_seed="1" * 32)
    assert res["passed"], res["failures"]
    assert res["detail"]["dists"] == cf.contract.input_dists
