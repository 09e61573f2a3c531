"""The sm100 architecture class and the B200 instance in the reference's hardware schema
(kta_b200/hardware/arch_sm100.yaml, model_b200_sm100.yaml): the reference's HwArch/HwModel
validation and MachineModel.build resolved them when tests/golden/hwarch.json was made; here
the files must still say what was resolved, every instance value must carry provenance, and
no operation class may list expected machine instructions (no reading of compiled code)."""

from __future__ import annotations

import json
from pathlib import Path

import yaml

HW = Path(__file__).resolve().parent.parent / "kta_b200" / "hardware"
GOLDEN = json.loads((Path(__file__).parent / "golden" / "hwarch.json").read_text())


def _load(name: str) -> dict:
    return yaml.safe_load((HW / name).read_text())


def test_arch_declares_what_the_reference_resolved():
    arch = _load("arch_sm100.yaml")
    assert f"{arch['name']}@{arch['version']}" == GOLDEN["arch"]
    assert sorted(r["name"] for r in arch["resources"]) == sorted(GOLDEN["resources"])
    assert sorted(o["name"] for o in arch["operation_classes"]) == GOLDEN["op_classes"]
    assert sorted(w["name"] for w in arch["walls"]) == sorted(GOLDEN["walls"])
    assert all("sass" not in o for o in arch["operation_classes"])


def test_instance_values_and_provenance():
    inst = _load("model_b200_sm100.yaml")
    arch = _load("arch_sm100.yaml")
    assert inst["arch"] == GOLDEN["arch"]
    assert set(arch["params"]) <= set(inst["limits"])
    keys = [f"peaks.{k}" for k in inst["peaks"]] + [f"limits.{k}" for k in inst["limits"]]
    assert all(k in inst["provenance"] for k in keys)
    for name, rate in inst["peaks"].items():
        assert GOLDEN["resources"][name]["rate"] == rate
        assert GOLDEN["resources"][name]["status"] == "measured"
    assert GOLDEN["scope_counts"] == {"chip": 1.0, "sm": 148.0, "smsp": 592.0}
    # the MUFU rate is the measured 16 ex2 per cycle per SM at the documented clock
    assert GOLDEN["resources"]["sfu"]["rate"] == 16 * 148 * inst["limits"]["sm_clock_hz"]
