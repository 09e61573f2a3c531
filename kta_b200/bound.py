"""Speed-of-light reporting: minimum work, per-resource bound, percentage of bound.

Follows the reference's semantics exactly:
- ``min_work``: ``Problem.params.min_work`` expressions over ``case.*`` evaluated per shape
  (src/kta/models/bound.py:42-53);
- ``sol_us``: each resource's work at its peak, in microseconds, skipping non-positive work
  (src/kta/models/l1.py:332-341, src/kta/models/machine.py:162-169);
- ``bound``: the largest per-resource time is the bound, its resource the bottleneck; a
  resource with work but no peak raises (bound.py:56-76);
- ``pct_of_bound = 100 * bound / best`` and ``near_bound`` when best <= 1.10 x bound
  (src/kta/orchestrator/analysis.py:33, :126-127, :140).

The B200 HwModel (kta_b200/hardware/model_b200.yaml) is a schema-1 model whose peaks are
the chip resources, as the reference resolves one without an HwArch
(src/kta/models/machine.py:278-298).
"""

from __future__ import annotations

import json
import os
from collections.abc import Mapping
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import yaml

from kta_b200.expr import Expr
from kta_b200.schemas import Bound, Problem

US_PER_S = 1e6
MIN_WORK_KEY = "min_work"
NEAR_BOUND = 1.10
HW_FILE = Path(__file__).resolve().parent / "hardware" / "model_b200.yaml"
ROOT = Path(__file__).resolve().parent.parent


class NotSupported(ValueError):
    pass


@dataclass(frozen=True)
class HwModel:
    target: str
    version: int
    peaks: dict[str, float]
    limits: dict[str, float] = field(default_factory=dict)
    sources: dict[str, str] = field(default_factory=dict)

    def rate(self, unit: str) -> float | None:
        p = self.peaks.get(unit)
        return float(p) if p is not None and p > 0 else None

    def time_s(self, unit: str, amount: float) -> float | None:
        r = self.rate(unit)
        return None if r is None else amount / r

    def to_yaml_body(self) -> dict[str, Any]:
        return {"target": self.target, "version": self.version, "peaks": dict(self.peaks),
                "limits": dict(self.limits)}


def load_model(path: str | Path = HW_FILE) -> HwModel:
    with open(path, encoding="utf-8") as f:
        doc = yaml.safe_load(f)
    peaks = {str(k): float(v) for k, v in (doc.get("peaks") or {}).items()}
    return HwModel(str(doc["target"]), int(doc["version"]), peaks,
                   {str(k): float(v) for k, v in (doc.get("limits") or {}).items()},
                   {k: "documented" for k in peaks})


def measured_peaks_path() -> Path:
    return Path(os.environ.get("KTA_MEASURED_PEAKS", ROOT / "MEASURED_PEAKS.json"))


def b200_model(measured: str | Path | None = None) -> HwModel:
    """The B200 model with the pod's measured copy bandwidth and cuBLAS bf16 throughput
    (MEASURED_PEAKS.json: hbm_gbs, bf16_tflops) replacing the documented dram and tensor
    peaks when the file exists. fp8 keeps its documented dense figure."""
    hw = load_model()
    path = Path(measured) if measured is not None else measured_peaks_path()
    if not path.exists():
        return hw
    data = json.loads(path.read_text(encoding="utf-8"))
    peaks = dict(hw.peaks)
    sources = dict(hw.sources)
    if data.get("hbm_gbs"):
        peaks["dram"] = float(data["hbm_gbs"]) * 1e9
        sources["dram"] = f"measured ({path.name}: hbm_gbs)"
    if data.get("bf16_tflops"):
        peaks["tensor"] = float(data["bf16_tflops"]) * 1e12
        sources["tensor"] = f"measured ({path.name}: bf16_tflops, burst)"
    return HwModel(hw.target, hw.version, peaks, hw.limits, sources)


def min_work(problem: Problem, shape: Mapping[str, Any]) -> dict[str, float]:
    raw = problem.params.get(MIN_WORK_KEY)
    if not isinstance(raw, dict) or not raw:
        raise NotSupported(
            f"case {problem.name}: params.{MIN_WORK_KEY} is missing (it maps each hardware unit "
            "to an expression of case.* values)"
        )
    return {str(u): float(Expr.parse(str(src), set()).eval({}, case=shape))
            for u, src in raw.items()}


def sol_us(work: Mapping[str, float], hw: HwModel) -> dict[str, float]:
    out: dict[str, float] = {}
    for r, w in sorted(work.items()):
        if w <= 0:
            continue
        s = hw.time_s(r, w)
        if s is not None:
            out[r] = s * US_PER_S
    return out


def bound(work: Mapping[str, float], hw: HwModel, case_name: str = "") -> Bound:
    missing = sorted(u for u, w in work.items() if w > 0 and hw.rate(u) is None)
    if missing:
        raise NotSupported(f"hardware model {hw.target}@{hw.version} gives no peak rate for "
                           f"{missing}")
    per_unit = sol_us(work, hw)
    if not per_unit:
        raise ValueError(f"case {case_name} declares no unit with positive work")
    bottleneck = max(per_unit, key=lambda u: (per_unit[u], u))
    return Bound(per_unit_us=per_unit, bound_us=per_unit[bottleneck], bottleneck=bottleneck)


def pct_of_bound(bound_us: float, best_us: float) -> float | None:
    return 100.0 * bound_us / best_us if best_us > 0 else None


def sol_report(problem: Problem, shape: Mapping[str, Any], best_us: float,
               hw: HwModel | None = None) -> dict[str, Any]:
    """The SOL columns of one measurement: bound, bottleneck, %SOL and per-unit
    achieved rates against the model's peaks."""
    hw = hw or b200_model()
    work = min_work(problem, shape)
    b = bound(work, hw, problem.name)
    rates = {u: w / (best_us / US_PER_S) for u, w in work.items() if w > 0}
    return {
        "bound_us": b.bound_us,
        "bottleneck": b.bottleneck,
        "per_unit_us": b.per_unit_us,
        "pct_of_bound": pct_of_bound(b.bound_us, best_us),
        "near_bound": best_us <= NEAR_BOUND * b.bound_us,
        "achieved": rates,
        "pct_of_peak": {u: 100.0 * r / hw.peaks[u] for u, r in rates.items() if u in hw.peaks},
        "peaks": {u: hw.peaks[u] for u in work if u in hw.peaks},
        "peak_sources": {u: hw.sources.get(u, "documented") for u in work if u in hw.peaks},
    }
