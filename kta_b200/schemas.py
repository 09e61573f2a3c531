"""Case records of KTA's evaluation schema, mirrored for the B200 path.

Field names, types and meanings follow src/kta/core/schemas/evaluation.py:13-131 (TensorSpec,
Problem, Contract, Case, Bound, Measurement, Check, Solution) and the strict record base of
src/kta/core/schemas/common.py:34-41 (unknown fields refused, frozen), so a case YAML written
for the reference validates here unchanged. ``CaseFile`` is the seed case format that
``kta case add`` reads (src/kta/cli/loop_cmds.py:57-88): problem, contract, case and an
optional library baseline.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any, Literal

import yaml
from pydantic import BaseModel, ConfigDict, Field, model_serializer

Unit = str


class Body(BaseModel):
    model_config = ConfigDict(extra="forbid", frozen=True)


class TensorSpec(Body):
    name: str
    shape: list[str] = Field(default_factory=list)
    dtype: str
    layout: str


class Problem(Body):
    name: str
    reference_impl: str
    inputs: list[TensorSpec] = Field(default_factory=list)
    outputs: list[TensorSpec] = Field(default_factory=list)
    params: dict[str, Any] = Field(default_factory=dict)


class Contract(Body):
    tolerances: dict[str, dict[str, Any]] = Field(default_factory=dict)
    input_dists: list[str] = Field(default_factory=list)
    edge_shapes: list[dict[str, Any]] = Field(default_factory=list)
    timing_boundary: str
    shape_scope: dict[str, Any] = Field(default_factory=dict)

    @model_serializer(mode="wrap")
    def _drop_undeclared_scope(self, handler: Any) -> dict[str, Any]:
        out: dict[str, Any] = handler(self)
        if not out.get("shape_scope"):
            out.pop("shape_scope", None)
        return out


class Case(Body):
    problem: str
    shape_dist: list[dict[str, Any]] = Field(default_factory=list)
    objective: Literal["weighted_latency", "max_normalized_latency"]
    target: str


class Build(Body):
    ok: bool
    regs: int | None = None
    spills: int | None = None
    smem: int | None = None
    log_summary: str


class Check(Body):
    passed: bool
    failures: list[dict[str, Any]] = Field(default_factory=list)


class Measurement(Body):
    median_us: float
    ci_low_us: float
    ci_high_us: float
    n: int
    clocks: dict[str, Any] = Field(default_factory=dict)
    temps: dict[str, Any] = Field(default_factory=dict)
    protocol: str


class Profile(Body):
    """Nsight Compute metrics of one launch (src/kta/core/schemas/evaluation.py:100-101)."""

    metrics: dict[str, float] = Field(default_factory=dict)


class Bound(Body):
    per_unit_us: dict[Unit, float] = Field(default_factory=dict)
    bound_us: float
    bottleneck: Unit


class Solution(Body):
    bucket: str | None = None
    assignment: dict[str, Any] = Field(default_factory=dict)
    pct_of_bound: float


class Baseline(Body):
    library: str
    call: str


class CaseFile(Body):
    """One seed case file: the three records plus the optional library baseline.

    ``entry`` (B200 addition) names the libkta_b200 C-ABI entry that implements the case."""

    problem: Problem
    contract: Contract
    case: dict[str, Any]
    baseline: Baseline | None = None
    entry: str | None = None

    def case_record(self, target: str = "b200") -> Case:
        body = {**self.case, "problem": self.problem.name, "target": self.case.get("target", target)}
        return Case.model_validate(body)


CASES_DIR = Path(__file__).resolve().parent / "cases"


def load_case_file(path: str | Path) -> CaseFile:
    p = Path(path)
    if not p.exists():
        p = CASES_DIR / f"{path}.yaml"
    with open(p, encoding="utf-8") as f:
        doc = yaml.safe_load(f)
    return CaseFile.model_validate(doc)


def case_names() -> list[str]:
    return sorted(p.stem for p in CASES_DIR.glob("*.yaml"))
