"""The check flow's shape selection without a GPU: hidden shapes and shape-scope gating must
equal the reference's own (`kta.checks.hidden.hidden_shapes`, `kta.checks.full.in_scope`,
recorded in tests/golden/hidden.json by make_golden.py); the private seed is kept private;
a sub-check that cannot run is a recorded failure, never a pass."""

from __future__ import annotations

import json
import stat
from pathlib import Path

import torch

from kta_b200 import checkflow, schemas

GOLDEN = json.loads((Path(__file__).parent / "golden" / "hidden.json").read_text())


def test_hidden_shapes_match_the_reference():
    assert len(GOLDEN["hidden"]) == 8
    for case in GOLDEN["hidden"]:
        got = checkflow.hidden_shapes(case["seed"], case["base"])
        assert [[s, c] for s, c in got] == case["shapes"]
        assert [c for _, c in got] == list(checkflow.HIDDEN_CATEGORIES)


def test_in_scope_matches_the_reference():
    for case in GOLDEN["scope"]:
        assert checkflow.in_scope(case["shape"], case["scope"], case["own"]) == case["in_scope"]


def test_private_seed_is_created_once_and_private(tmp_path):
    d = tmp_path / "checker"
    s1 = checkflow.private_seed(d)
    s2 = checkflow.private_seed(d)
    assert s1 == s2 and len(s1) == 32
    assert stat.S_IMODE((d / "hidden_seed").stat().st_mode) == 0o600


def test_every_case_file_selects_its_own_shapes():
    for name in schemas.case_names():
        cf = schemas.load_case_file(name)
        own = checkflow.case_shapes(cf)
        assert own, name
        assert all(checkflow.in_scope(s, cf.contract.shape_scope, own) for s in own)


def test_a_sub_check_that_cannot_run_fails_the_check(monkeypatch):
    from kta_b200 import checks

    def broken(*a, **k):
        raise RuntimeError("launch failed")

    monkeypatch.setattr(checks, "run_numeric", broken)
    cf = schemas.load_case_file("gemm_f16_1024")
    res = checkflow.quick_check(cf, {"M": 64, "N": 64, "K": 64})
    assert res["passed"] is False
    assert any(f["check"] == "numeric" and "launch failed" in f["error"]
               for f in res["failures"])
    assert set(res["skipped"]) == {"sanitizer", "sass"}
    if not torch.cuda.is_available():
        assert any(f["check"] == "anticheat" for f in res["failures"])
