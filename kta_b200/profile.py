"""Nsight Compute output ingested as KTA Profile records (src/kta/measure/profile.py).

- ``parse_ncu_csv(text, kernel)``: the reference's parser (profile.py:35-46): the CSV rows of
  ``ncu --csv`` output (lines starting with a quote; ncu's own ``==PROF==`` lines are
  skipped), only rows whose kernel name contains ``kernel``, ``Metric Value`` without
  thousands separators as a float, non-numeric values skipped with a warning; one value per
  metric name (the last row wins, as in the reference).
- ``profile_record``: those metrics as a ``Profile``; an ``ERR_NVGPUCTRPERM`` in the output
  (performance counters restricted to administrators) raises instead of returning partial
  numbers (profile.py:77-80).
- ``ncu_command``: the capture command of one launch (profile.py:58-67), always with
  ``--clock-control none`` so that the GPU's clocks are left as they are.
- ``launch_shares``: per kernel, the number of launches, their summed
  ``gpu__time_duration.sum`` and share of the total, from a launch-list capture (the tables of
  the profiles/ summaries).
"""

from __future__ import annotations

import csv
import io
import logging
from typing import Any

from kta_b200.schemas import Profile

log = logging.getLogger("kta_b200.profile")
DEFAULT_METRICS = [
    "gpu__time_duration.sum",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed",
]
NO_PERMISSION = "ERR_NVGPUCTRPERM"
_TIME_SCALE_US = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3,
                  "ms": 1e3, "second": 1e6, "s": 1e6}


class ProfilingNotPermitted(RuntimeError):
    pass


def _rows(text: str) -> list[dict[str, str]]:
    lines = [line for line in text.splitlines() if line.startswith('"')]
    return list(csv.DictReader(io.StringIO("\n".join(lines))))


def parse_ncu_csv(text: str, kernel: str) -> dict[str, float]:
    out: dict[str, float] = {}
    for row in _rows(text):
        if kernel not in (row.get("Kernel Name") or ""):
            continue
        value = (row.get("Metric Value") or "").replace(",", "")
        try:
            out[str(row["Metric Name"])] = float(value)
        except ValueError:
            log.warning("ncu metric %s has a non-numeric value %r", row.get("Metric Name"), value)
    return out


def profile_record(text: str, kernel: str, stderr: str = "") -> Profile:
    if NO_PERMISSION in text or NO_PERMISSION in stderr:
        raise ProfilingNotPermitted(
            "GPU performance counters are restricted to administrators (ncu ERR_NVGPUCTRPERM)")
    values = parse_ncu_csv(text, kernel)
    if not values:
        raise ValueError(f"ncu reported no metrics for kernel {kernel}")
    return Profile(metrics=values)


def ncu_command(program: list[str], kernel_regex: str, metrics: list[str] | None = None,
                skip: int = 0, count: int = 1, ncu: str = "ncu") -> list[str]:
    """``ncu --csv`` around ``program`` for ``count`` launches of the matching kernel after
    ``skip`` of them."""
    names = metrics or DEFAULT_METRICS
    return [ncu, "--csv", "--clock-control", "none", "--metrics", ",".join(names),
            "--kernel-name", f"regex:{kernel_regex}", "--launch-skip", str(skip),
            "--launch-count", str(count), *program]


def launch_shares(text: str) -> list[dict[str, Any]]:
    """Kernels of a ``gpu__time_duration.sum`` launch list, largest total first."""
    agg: dict[str, list[float]] = {}
    for row in _rows(text):
        if row.get("Metric Name") != "gpu__time_duration.sum":
            continue
        unit = (row.get("Metric Unit") or "").strip()
        if unit not in _TIME_SCALE_US:
            raise ValueError(f"unknown time unit {unit!r}")
        us = float((row.get("Metric Value") or "0").replace(",", "")) * _TIME_SCALE_US[unit]
        name = (row.get("Kernel Name") or "").split("(")[0].strip()
        acc = agg.setdefault(name, [0, 0.0])
        acc[0] += 1
        acc[1] += us
    total = sum(v[1] for v in agg.values())
    out = [{"kernel": k, "launches": int(v[0]), "total_us": v[1],
            "share": v[1] / total if total > 0 else 0.0} for k, v in agg.items()]
    return sorted(out, key=lambda r: -r["total_us"])
