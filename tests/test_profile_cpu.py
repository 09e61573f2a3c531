"""ncu output ingestion (kta_b200/profile.py) against the reference's own parser
(`kta.measure.profile.parse_ncu_csv`, recorded in tests/golden/ncu.json on a launch list
this build captured on a B200), the permission check and the capture command."""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from kta_b200 import profile

GOLDEN = Path(__file__).parent / "golden"
TEXT = (GOLDEN / "ncu_launches_decode.csv").read_text()


def test_parse_matches_the_reference():
    ref = json.loads((GOLDEN / "ncu.json").read_text())
    for kernel, metrics in ref.items():
        assert profile.parse_ncu_csv(TEXT, kernel) == pytest.approx(metrics), kernel


def test_profile_record_and_permission():
    rec = profile.profile_record(TEXT, "decode_kernel")
    assert rec.metrics["gpu__time_duration.sum"] > 0
    with pytest.raises(profile.ProfilingNotPermitted):
        profile.profile_record("==ERROR== ERR_NVGPUCTRPERM - no permission", "decode_kernel")
    with pytest.raises(ValueError):
        profile.profile_record(TEXT, "no_such_kernel")


def test_launch_shares_sum_to_one_and_lead_with_the_library_kernel():
    rows = profile.launch_shares(TEXT)
    assert rows[0]["kernel"].endswith("kta::decode_kernel<3, 1>")
    assert rows[0]["launches"] == 14
    assert sum(r["share"] for r in rows) == pytest.approx(1.0)


def test_capture_command_leaves_clocks_alone():
    cmd = profile.ncu_command(["python", "bench.py", "--profile"], "attn_fwd_kernel")
    i = cmd.index("--clock-control")
    assert cmd[i + 1] == "none"
    assert cmd[-3:] == ["python", "bench.py", "--profile"]
