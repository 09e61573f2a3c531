"""Correctness checks of a kernel case: numeric comparison, library-relative verdict,
NaN coverage, determinism and the linked-library scan.

Semantics follow the reference's checker:
- ``compare_output``: per element ``|y - ref| <= atol + rtol |ref|``; NaN where the reference
  is NaN and same-signed infinities match; relative L2 over finite elements; the count of
  non-finite outputs where the reference is finite (src/kta/checks/numeric.py:39-65);
- ``library_verdict``: a candidate passes at ``level`` when its relative L2 and largest
  absolute error stay within ``factor`` times the library's own, above small floors, with no
  non-finite output where the reference is finite (numeric.py:72-96);
- ``run_numeric``: one input set per distribution from the named stream
  ``checks.numeric:<shape json>:<dist>`` (numeric.py:121-124), outputs NaN-filled before the
  launch (src/kta/measure/bench.py:106-109), FP64 reference (and the library run when asked)
  through kta_b200.reference, failures recorded as the reference's Check record does
  (numeric.py:155-197);
- ``library_failures``: DT_NEEDED entries and undefined symbols of a module against the
  forbidden prefixes of src/kta/checks/anticheat.py:38-58.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Any

import numpy as np

from kta_b200.schemas import Check, Contract, Problem

FORBIDDEN_LIBS = ("libcublas", "libcudnn", "libtorch", "libc10", "libcufft", "libcurand",
                  "libcusparse", "libcusolver", "libnvinfer")
FORBIDDEN_SYMBOLS = ("cublas", "cudnn", "cufft", "curand", "cusparse", "cusolver", "_ZN2at",
                     "_ZN3c10")


class ConfigError(ValueError):
    pass


def canonical_json(obj: Any) -> str:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"), ensure_ascii=False)


# ---- element and L2 comparison ---------------------------------------------------------

def compare_output(got: np.ndarray, ref: np.ndarray, tol: dict[str, Any]) -> dict[str, Any]:
    with np.errstate(invalid="ignore", over="ignore"):
        g = np.asarray(got).astype(np.float64)
        r = np.asarray(ref, dtype=np.float64)
        nan_on_both = np.isnan(g) & np.isnan(r)
        inf_agrees = np.isinf(g) & np.isinf(r) & (np.sign(g) == np.sign(r))
        err = np.abs(g - r)
        ok = (err <= float(tol["atol"]) + float(tol["rtol"]) * np.abs(r)) | nan_on_both | inf_agrees
        finite = np.isfinite(r)
        diff = np.where(finite & np.isfinite(g), g - r, 0.0)
        ref_norm = float(np.linalg.norm(np.where(finite, r, 0.0)))
        dn = float(np.linalg.norm(diff))
        rel_l2 = dn / ref_norm if ref_norm > 0 else dn
        n_spurious = int(np.count_nonzero(~np.isfinite(g) & finite))
        return {
            "mismatches": int(np.count_nonzero(~ok)),
            "elements": int(g.size),
            "nan_count": int(np.count_nonzero(np.isnan(g) & ~np.isnan(r))),
            "nonfinite_where_ref_finite": n_spurious,
            "max_abs_err": float(np.max(np.where(finite & np.isfinite(g), err, 0.0),
                                        initial=0.0)),
            "rel_l2": rel_l2 if n_spurious == 0 else None,
        }


def relative_to_library(tol: dict[str, Any]) -> bool:
    return str(tol.get("relative_to", "")) == "library"


def library_verdict(stats: dict[str, Any], lib: dict[str, Any], tol: dict[str, Any],
                    level: str) -> tuple[bool, dict[str, Any]]:
    factor = float(tol.get(level, 2.0))
    rel_l2_min = float(tol.get("rel_l2_floor", 1e-6))
    abs_min = float(tol.get("abs_floor", 1e-3))
    l2_limit = max(factor * float(lib["rel_l2"] or 0.0), rel_l2_min)
    abs_limit = max(factor * float(lib["max_abs_err"]), abs_min)
    ok = (stats["nonfinite_where_ref_finite"] == 0 and stats["rel_l2"] is not None
          and stats["rel_l2"] <= l2_limit and stats["max_abs_err"] <= abs_limit)
    return ok, {
        "level": level,
        "factor": factor,
        "rel_l2_limit": l2_limit,
        "max_abs_limit": abs_limit,
        "library_rel_l2": lib["rel_l2"],
        "library_max_abs_err": lib["max_abs_err"],
        "library_mismatches": lib["mismatches"],
    }


def tolerance(contract: Contract, dtype: str) -> dict[str, Any]:
    if dtype not in contract.tolerances:
        raise ConfigError(f"the Contract has no tolerance for dtype {dtype}")
    return contract.tolerances[dtype]


def dists_for(contract: Contract, extra: list[str] | None) -> list[str]:
    out = list(dict.fromkeys([*contract.input_dists, *(extra or [])]))
    if not out:
        raise ConfigError("no input distributions: the Contract lists none")
    return out


def fixed_failed(stats: dict[str, Any], tol: dict[str, Any]) -> bool:
    limit = tol.get("rel_l2")
    l2 = stats["rel_l2"]
    return bool(stats["mismatches"]) or (limit is not None and (l2 is None or l2 > float(limit)))


# ---- the numeric check of one case on the GPU --------------------------------------------

def run_numeric(problem: Problem, contract: Contract, entry: str, shape: dict[str, Any],
                dists: list[str], seed: int = 0, level: str | None = None,
                repeat: int = 1) -> tuple[Check, list[dict[str, Any]]]:
    """Runs ``entry`` of libkta_b200 on one input set per distribution and compares every
    output with the FP64 reference; returns the Check record and per-output details.
    ``repeat`` > 1 also re-runs set 0 and requires byte-identical outputs (determinism)."""
    import torch

    from kta_b200 import inputs as kinp
    from kta_b200 import reference as kref
    from kta_b200 import runners

    failures: list[dict[str, Any]] = []
    details: list[dict[str, Any]] = []
    sets: list[dict[str, np.ndarray]] = []
    shapes: list[dict[str, Any]] = []
    for dist in dists:
        rng = kinp.named_rng(seed, f"checks.numeric:{canonical_json(shape)}:{dist}")
        full_shape, data = kinp.case_inputs(problem, shape, dist, rng)
        sets.append(data)
        shapes.append(full_shape)
    lib_wanted = level is not None and any(
        relative_to_library(tolerance(contract, o.dtype)) for o in problem.outputs)
    for i, dist in enumerate(dists):
        got = runners.run(entry, problem, shapes[i], sets[i], nan_fill=True)
        ref = kref.reference(problem, shapes[i], [sets[i]], library=lib_wanted)
        for t in problem.outputs:
            tol = tolerance(contract, t.dtype)
            stats = compare_output(got[t.name], ref.outputs[0][t.name], tol)
            extra: dict[str, Any] = {}
            if lib_wanted and relative_to_library(tol) and ref.library is not None:
                lib = compare_output(ref.library[0][t.name], ref.outputs[0][t.name], tol)
                ok, extra = library_verdict(stats, lib, tol, level or "loose")
                failed = not ok
            else:
                failed = fixed_failed(stats, tol)
            row = {"shape": shapes[i], "dist": dist, "output": t.name, **stats, **extra}
            details.append(row)
            if failed:
                failures.append({"check": "numeric", **row, "rtol": tol["rtol"],
                                 "atol": tol["atol"]})
    if repeat > 1:
        first = runners.run(entry, problem, shapes[0], sets[0], nan_fill=True, raw=True)
        for _ in range(repeat - 1):
            again = runners.run(entry, problem, shapes[0], sets[0], nan_fill=True, raw=True)
            for name in first:
                if not torch.equal(first[name].view(torch.uint8), again[name].view(torch.uint8)):
                    failures.append({"check": "determinism", "output": name,
                                     "shape": shapes[0]})
    return Check(passed=not failures, failures=failures), details


# ---- linked libraries (ELF dynamic section) ----------------------------------------------

def elf_dynamic(data: bytes) -> tuple[list[str], list[str]]:
    """DT_NEEDED entries and undefined dynamic symbols of an ELF64 little-endian module."""
    if data[:4] != b"\x7fELF" or data[4] != 2 or data[5] != 1:
        raise ConfigError("not a little-endian ELF64 module")
    shoff = struct.unpack_from("<Q", data, 0x28)[0]
    shentsize, shnum = struct.unpack_from("<HH", data, 0x3A)
    secs = [struct.unpack_from("<IIQQQQIIQQ", data, shoff + i * shentsize) for i in range(shnum)]
    needed: list[str] = []
    undefined: list[str] = []
    for sh in secs:
        sh_type, sh_offset, sh_size, sh_link, sh_entsize = sh[1], sh[4], sh[5], sh[6], sh[9]
        if sh_type == 6:  # SHT_DYNAMIC
            strtab = secs[sh_link]
            sbase = strtab[4]
            for off in range(sh_offset, sh_offset + sh_size, 16):
                tag, val = struct.unpack_from("<qQ", data, off)
                if tag == 0:
                    break
                if tag == 1:  # DT_NEEDED
                    end = data.index(b"\0", sbase + val)
                    needed.append(data[sbase + val:end].decode())
        if sh_type == 11 and sh_entsize:  # SHT_DYNSYM
            strtab = secs[sh_link]
            sbase = strtab[4]
            for off in range(sh_offset, sh_offset + sh_size, sh_entsize):
                name_off, info, other, shndx = struct.unpack_from("<IBBH", data, off)
                if shndx == 0 and name_off:
                    end = data.index(b"\0", sbase + name_off)
                    undefined.append(data[sbase + name_off:end].decode())
    return needed, undefined


def library_failures(path: str | Path) -> list[dict[str, Any]]:
    needed, undefined = elf_dynamic(Path(path).read_bytes())
    out: list[dict[str, Any]] = []
    for lib in needed:
        if lib.startswith(FORBIDDEN_LIBS):
            out.append({"check": "anticheat.library", "library": lib})
    for sym in undefined:
        if sym.startswith(FORBIDDEN_SYMBOLS):
            out.append({"check": "anticheat.symbol", "symbol": sym})
    return out
