"""The reference's measurement protocol (src/kta/measure/protocol.py:27-45, the `time` mode of
src/kta/measure/bench.py:124-192) run by kta_b200.measure.time_case on the fp16 GEMM 1024^3
case: >= 4 rotating input sets, NaN-filled outputs and a 2 x L2 flush before every launch, one
launch between two CUDA events, warm-up >= 10 iterations and 50 ms, >= 100 iterations and
200 ms, median with a bootstrap 95 % CI (src/kta/measure/stats.py:16-26)."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _sets(cf, shape, n):
    from kta_b200 import inputs as kinp

    return [kinp.case_inputs(cf.problem, shape, "normal_scaled",
                             kinp.named_rng(0, f"measure:{i}"))[1] for i in range(n)]


def test_time_case_gemm_f16_1024_median_and_ci(cuda_device):
    import torch

    from kta_b200 import measure, schemas

    cf = schemas.load_case_file("gemm_f16_1024")
    shape = {"M": 1024, "N": 1024, "K": 1024}
    res = measure.time_case(cf.entry, cf.problem, shape, _sets(cf, shape, 4))
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    assert res["flush_bytes"] == 2 * l2
    assert res["input_sets"] == 4
    assert res["n"] >= 100 and res["warmup_iters"] >= 10
    assert res["loop_s"] >= 0.2
    assert 0 < res["ci_low_us"] <= res["median_us"] <= res["ci_high_us"]
    # a 1024^3 f16 GEMM on a B200 takes microseconds, not milliseconds
    assert res["median_us"] < 200.0
    tflops = 2 * 1024 ** 3 / (res["median_us"] * 1e-6) / 1e12
    print(f"gemm_f16_1024 under the protocol: median {res['median_us']:.2f} us "
          f"[{res['ci_low_us']:.2f}, {res['ci_high_us']:.2f}] = {tflops:.1f} TFLOP/s")


def test_time_case_refuses_fewer_sets_than_the_protocol(cuda_device):
    from kta_b200 import measure, schemas

    cf = schemas.load_case_file("gemm_f16_1024")
    shape = {"M": 256, "N": 256, "K": 256}
    with pytest.raises(ValueError, match="input sets"):
        measure.time_case(cf.entry, cf.problem, shape, _sets(cf, shape, 2))
