"""Host-side mirror of KTA's case/checker API against the reference's own outputs
(tests/golden): input streams and generators, compare_output / library_verdict, min_work /
bound / pct_of_bound, case files. CPU only."""

from __future__ import annotations

import json
import random
from pathlib import Path

import numpy as np
import pytest

from kta_b200 import bound as kbound
from kta_b200 import checks, inputs, measure, schemas
from kta_b200.expr import Expr, ExprError
from kta_b200.schemas import Contract, Problem, TensorSpec

GOLDEN = Path(__file__).resolve().parent / "golden"


# ---- inputs ----------------------------------------------------------------------------

def test_generators_reproduce_the_reference_bytes():
    meta = json.loads((GOLDEN / "inputs.json").read_text())
    arrays = np.load(GOLDEN / "inputs.npz")
    for m in meta:
        rng = inputs.named_rng(m["seed"], m["stream"])
        spec = TensorSpec(name="A", shape=["M", "K"], dtype=m["dtype"], layout="row_major")
        got = inputs.generate(spec, m["shape"], m["dist"], rng)
        want = arrays[m["key"]]
        assert got.dtype == want.dtype and np.array_equal(got.view(np.uint8), want.view(np.uint8)), m


def test_one_stream_feeds_tensors_in_order():
    arrays = np.load(GOLDEN / "inputs.npz")
    for dtype in ("f16", "f32"):
        rng = inputs.named_rng(5, "pair")
        for t in ("A", "B"):
            spec = TensorSpec(name=t, shape=["M", "K"], dtype=dtype, layout="row_major")
            got = inputs.generate(spec, {"M": 5, "K": 6}, "normal", rng)
            assert np.array_equal(got, arrays[f"{dtype}_pair_{t}"])


def test_bf16_inputs_are_the_same_draw_rounded():
    spec16 = TensorSpec(name="A", shape=["n"], dtype="f32", layout="x")
    specbf = TensorSpec(name="A", shape=["n"], dtype="bf16", layout="x")
    a = inputs.generate(spec16, {"n": 64}, "normal", random.Random(3))
    b = inputs.generate(specbf, {"n": 64}, "normal", random.Random(3))
    assert b.dtype == np.uint16
    np.testing.assert_allclose(inputs.bf16_bits_to_f32(b), a, rtol=2 ** -8)


def test_unknown_distribution_is_refused():
    spec = TensorSpec(name="A", shape=["n"], dtype="f16", layout="x")
    with pytest.raises(inputs.NotSupported):
        inputs.generate(spec, {"n": 4}, "no_such_dist", random.Random(0))


def test_case_inputs_lengths_and_quantisation():
    dec = schemas.load_case_file("decode_gqa").problem
    shape, data = inputs.case_inputs(dec, {"B": 6, "Hq": 8, "Hkv": 2, "D": 128,
                                           "max_seqlen": 2000}, "normal", random.Random(1))
    ln, off = data["seqlens"], data["kv_offsets"]
    assert ln.dtype == np.int32 and off.dtype == np.int64
    assert ln.min() >= 1024 and ln.max() <= 2000
    assert shape["T"] == int(ln.sum()) and data["Kc"].shape == (shape["T"], 2, 128)
    assert np.array_equal(off, np.concatenate([[0], np.cumsum(ln)[:-1]]))
    fp8 = schemas.load_case_file("gemm_fp8_blockscaled").problem
    shape, data = inputs.case_inputs(fp8, {"M": 10, "N": 200, "K": 300}, "outliers",
                                     random.Random(2))
    assert data["A"].dtype == np.uint8 and data["sa"].shape == (10, 3)
    assert data["sb"].shape == (2, 3) and data["B"].shape == (200, 300)


# ---- compare_output / library_verdict ---------------------------------------------------

def test_compare_output_matches_reference():
    num = json.loads((GOLDEN / "numeric.json").read_text())
    for c in num["compare"]:
        got = np.array([float(v) for v in c["got"]])
        ref = np.array([float(v) for v in c["ref"]])
        out = checks.compare_output(got, ref, num["tol"])
        for k, v in c["out"].items():
            if isinstance(v, float):
                assert out[k] == pytest.approx(v, rel=1e-12, abs=0), (c["name"], k)
            else:
                assert out[k] == v, (c["name"], k)


def test_library_verdict_matches_reference():
    num = json.loads((GOLDEN / "numeric.json").read_text())
    for v in num["verdict"]:
        ok, detail = checks.library_verdict(v["cand"], v["lib"], v["tol"], v["level"])
        assert ok == v["ok"] and detail == v["detail"]


def test_dists_merge_and_refuse_empty():
    c = Contract(input_dists=["normal", "zeros"], timing_boundary="x")
    assert checks.dists_for(c, ["extreme", "normal"]) == ["normal", "zeros", "extreme"]
    with pytest.raises(checks.ConfigError):
        checks.dists_for(Contract(timing_boundary="x"), None)


# ---- SOL ------------------------------------------------------------------------------

def test_min_work_and_bound_match_reference():
    hw = kbound.load_model()
    for row in json.loads((GOLDEN / "bound.json").read_text()):
        prob = schemas.load_case_file(row["case"]).problem
        work = kbound.min_work(prob, row["shape"])
        assert work == pytest.approx(row["work"], rel=1e-12)
        b = kbound.bound(work, hw, row["case"])
        assert b.bottleneck == row["bottleneck"]
        assert b.bound_us == pytest.approx(row["bound_us"], rel=1e-12)
        assert b.per_unit_us == pytest.approx(row["per_unit_us"], rel=1e-12)


def test_bound_is_the_largest_unit_and_missing_peaks_raise():
    hw = kbound.HwModel("t", 1, {"dram": 2.5e11, "tensor": 2.0e14})
    b = kbound.bound({"dram": 2.5e5, "tensor": 2.0e8, "fma": 0.0}, hw)
    assert b.per_unit_us == pytest.approx({"dram": 1.0, "tensor": 1.0})
    with pytest.raises(kbound.NotSupported):
        kbound.bound({"l2": 1.0}, hw)
    assert kbound.pct_of_bound(10.0, 20.0) == 50.0


def test_measured_peaks_replace_documented_ones(tmp_path):
    p = tmp_path / "peaks.json"
    p.write_text(json.dumps({"hbm_gbs": 6000.0, "bf16_tflops": 1600.0}))
    hw = kbound.b200_model(p)
    assert hw.peaks["dram"] == 6.0e12 and hw.peaks["tensor"] == 1.6e15
    assert hw.peaks["tensor_fp8"] == 4.5e15
    assert "measured" in hw.sources["tensor"]


# ---- expressions, schemas, case files -------------------------------------------------

def test_expressions():
    assert Expr.parse("K // 2", {"K"}).eval({"K": 8}) == 4
    assert Expr.parse("ceil_div(K, 128)", {"K"}).eval({"K": 300}) == 3
    assert Expr.parse("2 * case.M * case.N", set()).eval({}, case={"M": 2, "N": 3}) == 12
    with pytest.raises(ExprError):
        Expr.parse("__import__('os')", set())
    with pytest.raises(ExprError):
        Expr.parse("M + X", {"M"})


def test_every_case_file_validates_in_the_reference_schema():
    for row in json.loads((GOLDEN / "schemas.json").read_text()):
        assert row["problem"] == row["contract"] == row["case_record"] == "ok", row
    for name in schemas.case_names():
        cf = schemas.load_case_file(name)
        assert cf.entry and cf.case_record().target == "b200"


def test_unknown_case_fields_are_refused():
    with pytest.raises(Exception):
        Problem.model_validate({"name": "x", "reference_impl": "y", "typo": 1})


# ---- measurement statistics -------------------------------------------------------------

def test_bootstrap_median_brackets_the_median_and_is_seeded():
    values = [10.0 + 0.01 * i for i in range(201)]
    med, lo, hi = measure.bootstrap_median(values, 1000, 0.95, random.Random(1))
    assert med == pytest.approx(11.0) and lo <= med <= hi and hi - lo < 0.5
    assert measure.bootstrap_median(values, 500, 0.95, random.Random(7)) == \
        measure.bootstrap_median(values, 500, 0.95, random.Random(7))


def test_significance_rule():
    v = measure.significance((99, 100), (104, 105), 0.05, 0.01, 3.0)
    assert v.significant and v.cis_disjoint and v.above_floor
    assert not measure.significance((99, 106), (104, 105), 0.05, 0.01, 3.0).significant


def test_protocol_refuses_unknown_params():
    with pytest.raises(ValueError):
        measure.MeasureParams.from_dict({"min_iters": 5, "lock_clocks_harder": True})
    assert measure.V1.l2_flush_factor == 2.0 and measure.V1.min_input_sets == 4


def test_library_scan_passes_on_the_built_library_and_flags_forbidden_names(tmp_path):
    from kta_b200 import lib

    assert checks.library_failures(lib.LIB_PATH) == []
    needed, _ = checks.elf_dynamic(lib.LIB_PATH.read_bytes())
    assert not any(n.startswith(("libcuda.", "libcublas", "libtorch")) for n in needed)
