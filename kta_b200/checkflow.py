"""The quick gate and the full check of a kernel case on libkta_b200, composed like the
reference's checker (src/kta/checks/full.py:109-224).

- ``quick_check`` (full.py:185-224): numeric on the entry as built, with the "normal"
  distribution when the contract lists it (QUICK_DISTS, full.py:41) else its first, at the
  loose library level; plus the anti-cheat checks.
- ``full_check`` (full.py:109-182): numeric over every distribution of the contract, the
  anti-cheat checks, the contract's edge shapes and three hidden shapes derived from a private
  seed (src/kta/checks/hidden.py:33-44: non-tile-multiple, unit-dimension, small-primes),
  each kept only when the contract's shape scope holds the kernel accountable for it
  (``in_scope``, full.py:70-87); the others are listed as out of scope.
- anti-cheat (src/kta/checks/anticheat.py): the kernels the entry launches must all be this
  library's (a CUPTI trace through torch.profiler in a fresh process stands in for the
  reference's nsys job);
  outputs are NaN-filled before the launch, so an unwritten element fails numeric; a second
  run of the same inputs must give the same bytes (determinism); the library must link none
  of the forbidden libraries (ELF dynamic section).
- compute-sanitizer is closed on this pool and SASS opcode checks are barred (no reading of
  compiled code): both are reported as skipped with the reason, never as passed.

The reference's record-store identity checks (full.py:49-67) compare a Case record with the
stored one; a case file here is a single record, so there is nothing to compare.

Each check returns ``{"passed", "failures", "sub_checks", "detail"}``; failures carry the
sub-check name like the reference's (``{"check": ..., "sub_check": ...}``).
"""

from __future__ import annotations

import hashlib
import os
import random
import secrets
from pathlib import Path
from typing import Any, Callable

from kta_b200 import checks
from kta_b200.schemas import CaseFile, Contract

QUICK_DISTS = ("normal",)
SMALL_PRIMES = (3, 5, 7, 11, 13, 17, 19, 23, 29, 31)
HIDDEN_CATEGORIES = ("non_tile_multiple", "unit_dimension", "small_primes")
KERNEL_PREFIXES = ("kta::",)  # every kernel of libkta_b200 lives in namespace kta
SKIPPED = {
    "sanitizer": "closed on this pool (compute-sanitizer); NaN-filled outputs, determinism "
                 "and device-side bounds checks stand in",
    "sass": "barred: no reading of compiled code",
}


# ---- hidden shapes (src/kta/checks/hidden.py) ----------------------------------------------
def private_seed(private_dir: str | Path | None = None) -> str:
    """The private seed of the hidden-shape check: drawn once from the OS, kept mode 600
    outside any workspace (hidden.py:24-31)."""
    d = Path(private_dir or os.environ.get("KTA_B200_CHECKER_DIR",
                                           Path.home() / ".kta_b200" / "checker"))
    path = d / "hidden_seed"
    if not path.exists():
        d.mkdir(parents=True, exist_ok=True, mode=0o700)
        path.write_text(secrets.token_hex(16), encoding="utf-8")
        path.chmod(0o600)
    return path.read_text(encoding="utf-8").strip()


def hidden_shapes(seed: str, base: dict[str, Any]) -> list[tuple[dict[str, Any], str]]:
    """One shape per category from the integer dimensions of ``base`` (hidden.py:33-44):
    every dimension moved off tile multiples, then one of them set to 1, then all set to
    small primes; drawn from sha256(seed:canonical base)."""
    digest = hashlib.sha256(f"{seed}:{checks.canonical_json(base)}".encode()).digest()
    rng = random.Random(int.from_bytes(digest[:8], "big"))
    dims = sorted(k for k, v in base.items() if isinstance(v, int) and not isinstance(v, bool))
    out: list[tuple[dict[str, Any], str]] = []
    if not dims:
        return out
    off = {k: max(1, int(base[k]) // 4 + rng.randrange(1, 16, 2)) for k in dims}
    out.append(({**base, **off}, "non_tile_multiple"))
    unit = rng.choice(dims)
    out.append(({**base, **{k: off[k] for k in dims}, unit: 1}, "unit_dimension"))
    out.append(({**base, **{k: rng.choice(SMALL_PRIMES) for k in dims}}, "small_primes"))
    return out


# ---- shape scope (full.py:70-87) ------------------------------------------------------------
def case_shapes(cf: CaseFile) -> list[dict[str, Any]]:
    return [dict(s.get("shape", {})) for s in cf.case.get("shape_dist", [])]


def in_scope(shape: dict[str, Any], scope: dict[str, Any],
             own: list[dict[str, Any]]) -> bool:
    """Whether the contract holds the kernel accountable for ``shape``: no scope = every
    shape; ``static`` = one of the case's own shapes; ``range`` = every ranged dimension
    inside its [lo, hi]."""
    kind = scope.get("kind")
    if not kind:
        return True
    dims = {k: v for k, v in shape.items() if isinstance(v, int) and not isinstance(v, bool)}
    if kind == "static":
        return any(all(s.get(k) == v for k, v in dims.items()) for s in own)
    if kind == "range":
        ranges: dict[str, Any] = scope.get("ranges") or {}
        return all(int(r[0]) <= dims[k] <= int(r[1]) for k, r in ranges.items() if k in dims)
    raise checks.ConfigError(f"shape_scope kind {kind!r} (expected static or range)")


# ---- sub-checks -------------------------------------------------------------------------------
def _numeric(cf: CaseFile, entry: str, shape: dict[str, Any], dists: list[str],
             level: str | None, label: str, seed: int) -> dict[str, Any]:
    chk, details = checks.run_numeric(cf.problem, cf.contract, entry, shape, dists, seed=seed,
                                      level=level)
    return {"name": label, "passed": chk.passed, "failures": list(chk.failures),
            "detail": {"shape": shape, "dists": dists, "level": level, "rows": details}}


def _anticheat(cf: CaseFile, entry: str, shape: dict[str, Any], seed: int) -> dict[str, Any]:
    """Kernels launched, determinism (NaN coverage is part of numeric) and libraries."""
    import torch

    from kta_b200 import inputs as kinp
    from kta_b200 import lib, runners

    failures: list[dict[str, Any]] = []
    rng = kinp.named_rng(seed, f"checks.anticheat:{checks.canonical_json(shape)}")
    full_shape, data = kinp.case_inputs(cf.problem, shape, "normal", rng)
    names = runners.trace_kernels(entry, cf.problem, full_shape, data)
    first = runners.run(entry, cf.problem, full_shape, data, nan_fill=True, raw=True)
    foreign = sorted({n for n in names if not any(k in n for k in KERNEL_PREFIXES)})
    if not names:
        failures.append({"check": "anticheat.kernels", "detail": "no kernel launched"})
    for n in foreign:
        failures.append({"check": "anticheat.kernels", "detail": f"undeclared kernel {n}"})
    again = runners.run(entry, cf.problem, full_shape, data, nan_fill=True, raw=True)
    for name in first:
        a, b = first[name].contiguous(), again[name].contiguous()
        if a.shape != b.shape or not torch.equal(a.view(torch.uint8), b.view(torch.uint8)):
            failures.append({"check": "anticheat.determinism", "output": name})
    for f in checks.library_failures(lib.LIB_PATH):
        failures.append({"check": "anticheat.libraries", **f})
    return {"name": "anticheat", "passed": not failures, "failures": failures,
            "detail": {"kernels": sorted(set(names)), "shape": full_shape}}


def _compose(subs: list[dict[str, Any]], errors: list[dict[str, Any]],
             detail: dict[str, Any]) -> dict[str, Any]:
    failures = list(errors)
    for s in subs:
        failures += [{**f, "sub_check": s["name"]} for f in s["failures"]]
    return {"passed": not failures and bool(subs), "failures": failures,
            "sub_checks": {s["name"]: s["passed"] for s in subs},
            "skipped": dict(SKIPPED), "detail": detail}


def _guarded(name: str, fn: Callable[[], dict[str, Any]], subs: list[dict[str, Any]],
             errors: list[dict[str, Any]]) -> None:
    """A sub-check that cannot run (the library refuses the shape, a launch fails) is a
    failure of the whole check, recorded under its name (full.py:135-139)."""
    try:
        subs.append(fn())
    except Exception as exc:  # noqa: BLE001 - every error becomes a recorded failure
        errors.append({"check": name, "error": f"{type(exc).__name__}: {exc}"})


def quick_check(cf: CaseFile, shape: dict[str, Any] | None = None, *,
                entry: str | None = None, level: str = "loose",
                seed: int = 0) -> dict[str, Any]:
    """The gate before measuring: cheap, on the entry as built, no other shapes."""
    entry = entry or cf.entry
    shape = shape or case_shapes(cf)[0]
    contract: Contract = cf.contract
    wanted = [d for d in QUICK_DISTS if d in contract.input_dists]
    dists = wanted or checks.dists_for(contract, None)[:1]
    subs: list[dict[str, Any]] = []
    errors: list[dict[str, Any]] = []
    _guarded("numeric", lambda: _numeric(cf, entry, shape, dists, level, "numeric", seed),
             subs, errors)
    _guarded("anticheat", lambda: _anticheat(cf, entry, shape, seed), subs, errors)
    return _compose(subs, errors, {"dists": dists, "level": level, "shape": shape})


def full_check(cf: CaseFile, shape: dict[str, Any] | None = None, *,
               entry: str | None = None, level: str | None = None,
               extra_dists: list[str] | None = None, hidden_seed: str | None = None,
               seed: int = 0) -> dict[str, Any]:
    """Numeric on every distribution, anti-cheat, edge shapes and in-scope hidden shapes."""
    entry = entry or cf.entry
    shape = shape or case_shapes(cf)[0]
    contract: Contract = cf.contract
    dists = checks.dists_for(contract, extra_dists)
    subs: list[dict[str, Any]] = []
    errors: list[dict[str, Any]] = []
    _guarded("numeric", lambda: _numeric(cf, entry, shape, dists, level, "numeric", seed),
             subs, errors)
    _guarded("anticheat", lambda: _anticheat(cf, entry, shape, seed), subs, errors)
    others: list[tuple[dict[str, Any], str | None]] = [(dict(e), None)
                                                        for e in contract.edge_shapes]
    hseed = hidden_seed if hidden_seed is not None else private_seed()
    others += [(s, cat) for s, cat in hidden_shapes(hseed, shape)]
    scope, own = contract.shape_scope, case_shapes(cf)
    skipped = [cat or "edge" for s, cat in others if not in_scope(s, scope, own)]
    others = [(s, cat) for s, cat in others if in_scope(s, scope, own)]
    for other, category in others:
        label = "numeric.edge" if category is None else f"numeric.hidden.{category}"
        _guarded(label, lambda o=other, lb=label: _numeric(cf, entry, o, dists, level, lb, seed),
                 subs, errors)
    return _compose(subs, errors, {"dists": dists, "level": level, "shape": shape,
                                   "hidden_shapes": len(others), "out_of_scope": skipped,
                                   "shape_scope": scope})
