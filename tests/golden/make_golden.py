"""Generates the golden fixtures of tests/golden from the reference's own Python code.

Run in a container where the reference (kernel-template-agent) is checked out; it is not
needed afterwards (the fixtures are committed):

    python tests/golden/make_golden.py <path of the kernel-template-agent checkout>

What it records, each from the reference itself:
- inputs.npz: `kta.measure.inputs.generate` draws for every distribution of
  `kta.checks.inputs.TABLE`, f16 and f32, from named streams `Context.rng` derives;
- numeric.json: `kta.checks.numeric.compare_output` and `library_verdict` on fixed cases;
- bound.json: `kta.models.bound.min_work` / `bound` on the B200 case files with the B200
  HwModel (kta_b200/hardware/model_b200.yaml) resolved by the reference's MachineModel;
- statements.npz: the reference's statement runner `src/kta/checks/scripts/ref_torch.py`,
  run unmodified except for its device ("cuda" -> "cpu", the final cuda sync dropped), on
  inputs from the
  reference's generator: FP64 and "library" outputs of the GEMM statements (the seed
  cases' `C = A @ B` and the B200 `C = A @ B.T`), the causal attention, decode and FP8
  statements of kta_b200/cases (small shapes);
- schemas.json: whether each kta_b200 case file's problem / contract / case validate in
  the reference's pydantic records;
- hidden.json: `kta.checks.hidden.hidden_shapes` for fixed seeds and base shapes, and
  `kta.checks.full.in_scope` on static, range and unscoped contracts;
- hwarch.json: kta_b200/hardware/arch_sm100.yaml and model_b200_sm100.yaml validated as the
  reference's HwArch and HwModel and resolved by its `MachineModel.build`: each resource's
  rate and status, the walls' limits and the operation classes;
- ncu.json: `kta.measure.profile.parse_ncu_csv` on ncu_launches_decode.csv (a launch list
  this build captured on a B200 with `ncu --csv`) for several kernel names.
"""

from __future__ import annotations

import json
import random
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import yaml

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def main(ref_root: str) -> int:
    ref = Path(ref_root)
    sys.path.insert(0, str(ref / "src"))
    from kta.checks import inputs as cinputs
    from kta.checks import numeric
    from kta.core.context import Context
    from kta.core.schemas.evaluation import Case, Contract, Problem, TensorSpec
    from kta.core.schemas.hardware import HwModel
    from kta.measure import inputs as minputs
    import importlib

    mbound = importlib.import_module("kta.models.bound")

    # ---- named streams and generators ----
    arrays: dict[str, np.ndarray] = {}
    meta = []
    for dtype in ("f16", "f32"):
        for dist in sorted(cinputs.TABLE):
            for shape in ({"M": 4, "K": 8}, {"M": 3, "K": 7}):
                name = f"checks.numeric:{json.dumps(shape, sort_keys=True)}:{dist}"
                rng = Context.rng(SimpleNamespace(seed=11), name)
                spec = TensorSpec(name="A", shape=["M", "K"], dtype=dtype, layout="row_major")
                x = minputs.generate(spec, shape, dist, rng, cinputs.TABLE)
                key = f"{dtype}_{dist}_{shape['M']}x{shape['K']}"
                arrays[key] = x
                meta.append({"key": key, "dtype": dtype, "dist": dist, "shape": shape,
                             "seed": 11, "stream": name})
        # two tensors drawn one after the other from one stream (random_inputs order)
        rng = Context.rng(SimpleNamespace(seed=5), "pair")
        for t in ("A", "B"):
            spec = TensorSpec(name=t, shape=["M", "K"], dtype=dtype, layout="row_major")
            arrays[f"{dtype}_pair_{t}"] = minputs.generate(spec, {"M": 5, "K": 6}, "normal", rng)
    np.savez(HERE / "inputs.npz", **arrays)
    (HERE / "inputs.json").write_text(json.dumps(meta, indent=1))

    # ---- compare_output / library_verdict ----
    tol = {"rtol": 1e-2, "atol": 1e-2, "rel_l2": 1e-3}
    g = np.random.default_rng(3)
    cases = []
    refv = np.linspace(-4, 4, 100)
    got = refv.astype(np.float16)
    cases.append(("rounding", got.astype(np.float64), refv))
    bad = got.astype(np.float64).copy()
    bad[-10:] = np.nan
    cases.append(("unwritten", bad, refv))
    cases.append(("nan_inf", np.array([np.nan, np.inf, 1.0]), np.array([np.nan, np.inf, 1.0])))
    r2 = g.standard_normal(257)
    cases.append(("noisy", r2 + g.standard_normal(257) * 3e-3, r2))
    cases.append(("inf_mismatch", np.array([np.inf, -np.inf, 2.0]), np.array([np.inf, np.inf, 2.0])))
    num = {"tol": tol, "compare": [], "verdict": []}
    for name, gg, rr in cases:
        num["compare"].append({"name": name, "got": [repr(float(v)) for v in gg],
                               "ref": [repr(float(v)) for v in rr],
                               "out": numeric.compare_output(np.asarray(gg), np.asarray(rr), tol)})
    vt = {"rtol": 0.01, "atol": 0.01, "relative_to": "library", "loose": 4.0, "strict": 1.5}

    def st(l2, mx, nf=0):
        return {"rel_l2": l2, "max_abs_err": mx, "mismatches": 480, "nonfinite_where_ref_finite": nf}

    for cand, lib in [((2.1e-4, 8.06), (1.9e-4, 7.5)), ((0.3, 900.0), (1.9e-4, 7.5)),
                      ((3.8e-4, 15.0), (1.9e-4, 7.5)), ((5e-7, 5e-4), (0.0, 0.0)),
                      ((1e-3, 0.5), (0.0, 0.0))]:
        for level in ("loose", "strict"):
            ok, detail = numeric.library_verdict(st(*cand), st(*lib), vt, level)
            num["verdict"].append({"cand": st(*cand), "lib": st(*lib), "tol": vt, "level": level,
                                   "ok": ok, "detail": detail})
    ok, detail = numeric.library_verdict(st(1e-5, 0.1, 3), st(1.9e-4, 7.5), vt, "loose")
    num["verdict"].append({"cand": st(1e-5, 0.1, 3), "lib": st(1.9e-4, 7.5), "tol": vt,
                           "level": "loose", "ok": ok, "detail": detail})
    (HERE / "numeric.json").write_text(json.dumps(num, indent=1))

    # ---- min_work / bound with the B200 HwModel ----
    hwdoc = yaml.safe_load((REPO / "kta_b200" / "hardware" / "model_b200.yaml").read_text())
    hw = HwModel.model_validate(hwdoc)
    bounds = []
    for path in sorted((REPO / "kta_b200" / "cases").glob("*.yaml")):
        doc = yaml.safe_load(path.read_text())
        prob = Problem.model_validate(doc["problem"])
        case = Case.model_validate({**doc["case"], "problem": prob.name, "target": "b200"})
        for item in case.shape_dist:
            shape = dict(item["shape"])
            if "T" in str(doc["problem"]["params"]["min_work"]):
                shape["T"] = 294912  # a fixed total KV length for the decode case
            work = mbound.min_work(prob, shape)
            b = mbound.bound(case, shape, hw, work)
            bounds.append({"case": path.stem, "shape": shape, "work": work,
                           "per_unit_us": b.per_unit_us, "bound_us": b.bound_us,
                           "bottleneck": b.bottleneck})
    (HERE / "bound.json").write_text(json.dumps(bounds, indent=1))

    # ---- schemas ----
    schemas = []
    for path in sorted((REPO / "kta_b200" / "cases").glob("*.yaml")):
        doc = yaml.safe_load(path.read_text())
        res = {"case": path.stem}
        for key, model in (("problem", Problem), ("contract", Contract)):
            try:
                model.model_validate(doc[key])
                res[key] = "ok"
            except Exception as exc:  # noqa: BLE001 - recorded as the fixture
                res[key] = f"error: {type(exc).__name__}"
        try:
            Case.model_validate({**doc["case"], "problem": "p", "target": "b200"})
            res["case_record"] = "ok"
        except Exception as exc:  # noqa: BLE001
            res["case_record"] = f"error: {type(exc).__name__}"
        schemas.append(res)
    (HERE / "schemas.json").write_text(json.dumps(schemas, indent=1))

    # ---- hidden shapes and shape scope (the full check's shape selection) ----
    from kta.checks import hidden as chidden
    from kta.checks.full import in_scope as ref_in_scope

    hidden_cases = []
    for seed in ("0123456789abcdef0123456789abcdef", "feedface" * 4):
        for base in ({"M": 8192, "N": 8192, "K": 8192}, {"M": 16, "N": 8192, "K": 8192},
                     {"B": 8, "H": 32, "S": 4096, "D": 128}, {"M": 1024, "N": 1024, "K": 1024,
                                                            "dtype": "f16"}):
            got = chidden.hidden_shapes(seed, base)
            hidden_cases.append({"seed": seed, "base": base,
                                 "shapes": [[s, c] for s, c in got]})
    scopes = []
    own = [{"M": 64, "N": 64, "K": 64}, {"M": 128, "N": 256, "K": 64}]
    for scope in ({}, {"kind": "static"}, {"kind": "range", "ranges": {"M": [1, 100]}},
                  {"kind": "range", "ranges": {"M": [1, 4096], "K": [64, 64]}}):
        for shape in ({"M": 64, "N": 64, "K": 64}, {"M": 65, "N": 64, "K": 64},
                      {"M": 128, "N": 256, "K": 64}, {"M": 3, "N": 5, "K": 7}):
            scopes.append({"scope": scope, "own": own, "shape": shape,
                           "in_scope": ref_in_scope(shape, scope, own)})
    (HERE / "hidden.json").write_text(json.dumps({"hidden": hidden_cases, "scope": scopes},
                                                 indent=1))

    # ---- the sm100 architecture class and the B200 instance in the reference's schema ----
    from kta.core.schemas.hwmodel import HwArch
    from kta.models.machine import MachineModel

    hw_dir = REPO / "kta_b200" / "hardware"
    arch = HwArch.model_validate(yaml.safe_load((hw_dir / "arch_sm100.yaml").read_text()))
    inst = HwModel.model_validate(yaml.safe_load((hw_dir / "model_b200_sm100.yaml").read_text()))
    mm = MachineModel.build(inst, arch)
    hwrec = {
        "arch": arch.ref,
        "resources": {k: {"rate": r.rate, "status": r.status, "scope": r.scope,
                          "amount": r.amount} for k, r in sorted(mm.resources.items())},
        "walls": {w.spec.name: w.limit for w in mm.walls},
        "op_classes": sorted(mm.op_classes),
        "scope_counts": dict(mm.scope_counts),
    }
    (HERE / "hwarch.json").write_text(json.dumps(hwrec, indent=1))

    # ---- ncu CSV ingestion ----
    from kta.measure.profile import parse_ncu_csv

    text = (HERE / "ncu_launches_decode.csv").read_text()
    parsed = {k: parse_ncu_csv(text, k) for k in ("decode_kernel", "kta::", "FillFunctor",
                                                  "no_such_kernel", "")}
    (HERE / "ncu.json").write_text(json.dumps(parsed, indent=1, sort_keys=True))

    # ---- the reference's statement runner on the CPU ----
    script_src = (ref / "src" / "kta" / "checks" / "scripts" / "ref_torch.py").read_text()
    if script_src.count('"cuda"') != 2 or script_src.count("torch.cuda.synchronize()") != 1:
        raise SystemExit("ref_torch.py changed: expected two \"cuda\" devices and one sync")
    work_dir = Path(tempfile.mkdtemp(prefix="kta_golden_"))
    cpu_src = script_src.replace('"cuda"', '"cpu"').replace("torch.cuda.synchronize()", "None")
    (work_dir / "ref_torch_cpu.py").write_text(cpu_src)
    (work_dir / "in").mkdir()
    (work_dir / "out").mkdir()

    def run(tag, statement, shape, tensors, outputs, library=True):
        files = {}
        for name, arr in tensors.items():
            p = work_dir / "in" / f"{tag}_{name}.bin"
            arr.tofile(p)
            files[name] = str(p)
        spec = {"statement": statement, "compute": "f64", "shape": shape,
                "inputs": {n: {"dtype": a.dtype.name, "dims": list(a.shape)}
                           for n, a in tensors.items()},
                "outputs": outputs, "sets": [files], "library": library}
        (work_dir / "ref.json").write_text(json.dumps(spec))
        subprocess.run([sys.executable, "ref_torch_cpu.py", "ref.json"], cwd=work_dir,
                       check=True)
        res = {}
        for o in outputs:
            res[f"{tag}.{o}.f64"] = np.fromfile(work_dir / "out" / f"{o}.s0.bin")
            if library:
                res[f"{tag}.{o}.lib"] = np.fromfile(work_dir / "out" / f"{o}.lib.s0.bin")
        return res

    st_out: dict[str, np.ndarray] = {}
    rng = Context.rng(SimpleNamespace(seed=7), "golden.statements")

    def gen(name, dims_shape, dtype, dist="normal"):
        spec = TensorSpec(name=name, shape=list(dims_shape), dtype=dtype, layout="row_major")
        return minputs.generate(spec, dict(dims), dist, rng, cinputs.TABLE)

    dims = {"M": 24, "N": 40, "K": 56}
    a = gen("A", ["M", "K"], "f16")
    bkn = gen("B", ["K", "N"], "f16")
    bnk = gen("B", ["N", "K"], "f16")
    st_out.update({"nn.A": a, "nn.B": bkn, "tn.B": bnk})
    st_out.update(run("nn", "C = A @ B", dims, {"A": a, "B": bkn}, ["C"]))
    st_out.update(run("tn", "C = A @ B.T", dims, {"A": a, "B": bnk}, ["C"]))

    def case_statement(name):
        return yaml.safe_load((REPO / "kta_b200" / "cases" / f"{name}.yaml").read_text())[
            "problem"]["reference_impl"]

    dims = {"B": 2, "S": 24, "H": 3, "D": 16}
    q = gen("Q", ["B", "S", "H", "D"], "f32")
    k = gen("K", ["B", "S", "H", "D"], "f32")
    v = gen("V", ["B", "S", "H", "D"], "f32")
    st_out.update({"attn.Q": q, "attn.K": k, "attn.V": v})
    st_out.update(run("attn", case_statement("attn_causal"), dims, {"Q": q, "K": k, "V": v},
                      ["O", "LSE"], library=False))

    lengths = np.array([5, 17, 1], dtype=np.int32)
    offsets = np.array([0, 5, 22], dtype=np.int64)
    dims = {"B": 3, "Hq": 8, "Hkv": 2, "D": 16, "T": 23}
    qd = gen("Q", ["B", "Hq", "D"], "f32")
    kc = gen("Kc", ["T", "Hkv", "D"], "f32")
    vc = gen("Vc", ["T", "Hkv", "D"], "f32")
    st_out.update({"dec.Q": qd, "dec.Kc": kc, "dec.Vc": vc, "dec.seqlens": lengths,
                   "dec.offsets": offsets})
    st_out.update(run("dec", case_statement("decode_gqa"), dims,
                      {"Q": qd, "Kc": kc, "Vc": vc, "seqlens": lengths, "kv_offsets": offsets},
                      ["O"], library=False))

    dims = {"M": 6, "N": 136, "K": 160}
    # dequantised-statement check: e4m3 codes are passed as their f32 values
    af = gen("A", ["M", "K"], "f32")
    bf = gen("B", ["N", "K"], "f32")
    sa = np.abs(gen("sa", ["M", "2"], "f32")).astype(np.float32) + np.float32(0.5)
    sb = np.abs(gen("sb", ["2", "2"], "f32")).astype(np.float32) + np.float32(0.5)
    st_out.update({"fp8.A": af, "fp8.B": bf, "fp8.sa": sa, "fp8.sb": sb})
    st_out.update(run("fp8", case_statement("gemm_fp8_blockscaled"), dims,
                      {"A": af, "sa": sa, "B": bf, "sb": sb}, ["C"], library=False))
    dims = {"M": 12, "N": 40}
    xr = gen("X", ["M", "N"], "f16")
    wr = gen("W", ["N"], "f16")
    st_out.update({"rms.X": xr, "rms.W": wr})
    st_out.update(run("rms", case_statement("rmsnorm_f16"), dims, {"X": xr, "W": wr}, ["Y"],
                      library=False))
    xs = gen("X", ["M", "N"], "f16", dist="large_dynamic_range")
    st_out.update({"smax.X": xs})
    st_out.update(run("smax", case_statement("softmax_f16"), dims, {"X": xs}, ["Y"],
                      library=False))
    dims = {"E": 3, "T": 12, "N": 20, "K": 24}
    am = gen("A", ["T", "K"], "f16")
    wm = gen("W", ["E", "K", "N"], "f16")
    st_out.update({"moe.A": am, "moe.W": wm})
    st_out.update(run("moe", case_statement("moe_gemm_f16"), dims, {"A": am, "W": wm}, ["C"],
                      library=False))
    sys.path.insert(0, str(REPO))
    from kta_b200.inputs import quantize_4bit

    dims = {"M": 6, "N": 10, "K": 64}
    a4 = gen("A", ["M", "K"], "f16")
    src = gen("Bsrc", ["N", "K"], "f32")
    for tag, fmt, grp, case in (("w4", "int4", 32, "w4gemm_f16"),
                                ("nvfp4", "e2m1", 16, "nvfp4gemm_f16")):
        bq, sc = quantize_4bit(src, fmt, grp)
        st_out.update({f"{tag}.A": a4, f"{tag}.Bq": bq, f"{tag}.Sc": sc})
        st_out.update(run(tag, case_statement(case), dims, {"A": a4, "Bq": bq, "Sc": sc}, ["C"],
                          library=False))
    np.savez(HERE / "statements.npz", **st_out)
    shutil.rmtree(work_dir)
    print("wrote", sorted(p.name for p in HERE.iterdir()))
    return 0


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <kernel-template-agent "
                         "checkout>")
    sys.exit(main(sys.argv[1]))
