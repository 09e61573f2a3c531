"""Runs a case's libkta_b200 entry on host input sets, the way the reference's bench job
runs a module (src/kta/measure/bench.py:56-78, :111-122): inputs copied to the device,
outputs allocated and NaN-filled (all-ones bytes) before the launch, one launch, a
synchronisation, outputs copied back. Every entry goes through the C ABI (kta_b200.ops)."""

from __future__ import annotations

from typing import Any, Callable

import numpy as np
import torch

from kta_b200 import ops
from kta_b200.reference import to_torch
from kta_b200.schemas import Problem

NAN_BYTE = 0xFF


def _gemm(entry: str) -> Callable[..., dict[str, torch.Tensor]]:
    layout = "kn" if "_nn_" in entry else "nk"

    def run(t: dict[str, torch.Tensor], shape: dict[str, Any], out: dict[str, torch.Tensor]):
        return {"C": ops.gemm(t["A"], t["B"], out=out["C"], b_layout=layout)}

    return run


def _fp8(t, shape, out):
    return {"C": ops.gemm_fp8_blockscaled(t["A"], t["sa"], t["B"], t["sb"], out=out["C"])}


def _attn(t, shape, out):
    o, lse = ops.attn_fwd_causal(t["Q"], t["K"], t["V"], scale=shape["D"] ** -0.5,
                                 out=out["O"], lse=out["LSE"])
    return {"O": o, "LSE": lse}


def _decode(t, shape, out):
    # max_seqlen comes from the host (run() fills it in): a device reduction here would be a
    # kernel outside the library inside the entry's launch
    return {"O": ops.decode_gqa(t["Q"], t["Kc"], t["Vc"], t["seqlens"], t["kv_offsets"],
                                int(shape["max_seqlen"]), scale=shape["D"] ** -0.5,
                                out=out["O"])}


def _w4(t, shape, out):
    return {"C": ops.gemm_4bit(t["A"], t["Bq"], t["Sc"], "int4", 32, out=out["C"])}


def _nvfp4(t, shape, out):
    return {"C": ops.gemm_4bit(t["A"], t["Bq"], t["Sc"], "e2m1", 16, out=out["C"])}


def _moe(t, shape, out):
    return {"C": ops.moe_gemm(t["A"], t["W"], out=out["C"])}


def _rms(t, shape, out):
    return {"Y": ops.rmsnorm(t["X"], t["W"], eps=1e-6, out=out["Y"])}


def _softmax(t, shape, out):
    return {"Y": ops.softmax(t["X"], out=out["Y"])}


RUNNERS: dict[str, Callable[..., dict[str, torch.Tensor]]] = {
    "kta_gemm_w4a16_f16": _w4,
    "kta_gemm_nvfp4_f16": _nvfp4,
    "kta_moe_gemm_f16": _moe,
    "kta_moe_gemm_bf16": _moe,
    "kta_rmsnorm_f16": _rms,
    "kta_rmsnorm_bf16": _rms,
    "kta_softmax_f16": _softmax,
    "kta_softmax_bf16": _softmax,
    "kta_gemm_bf16": _gemm("kta_gemm_bf16"),
    "kta_gemm_f16": _gemm("kta_gemm_f16"),
    "kta_gemm_nn_bf16": _gemm("kta_gemm_nn_bf16"),
    "kta_gemm_nn_f16": _gemm("kta_gemm_nn_f16"),
    "kta_gemm_fp8_blockscaled": _fp8,
    "kta_attn_fwd_causal_bf16": _attn,
    "kta_decode_gqa_bf16": _decode,
}

_TORCH = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32,
          "e4m3": torch.float8_e4m3fn, "i32": torch.int32, "i64": torch.int64,
          "i8": torch.int8}


def resolve(entry: str) -> Callable[..., dict[str, torch.Tensor]]:
    """The runner of ``entry``: a libkta_b200 entry name from RUNNERS, or a plug-in runner
    named ``"package.module:function"`` with the same ``(inputs, shape, outputs) -> outputs``
    signature, imported on first use (so the checker can check a caller's own launch code the
    way the reference's checker checks any built module)."""
    if entry in RUNNERS:
        return RUNNERS[entry]
    if ":" in entry:
        import importlib

        mod, _, name = entry.partition(":")
        fn = getattr(importlib.import_module(mod), name, None)
        if callable(fn):
            return fn
    raise ValueError(f"no runner for entry {entry!r}")


def run(entry: str, problem: Problem, shape: dict[str, Any], data: dict[str, np.ndarray],
        nan_fill: bool = True, raw: bool = False, device: str = "cuda",
        launched: list[str] | None = None) -> dict[str, Any]:
    """Outputs of one launch as float64 numpy arrays (``raw``: device tensors). With
    ``launched``, the names of the GPU kernels the entry itself launched are appended to it
    (a CUPTI trace through torch.profiler around the launch only; memsets and copies are not
    kernels)."""
    from kta_b200 import inputs as kinp

    fn = resolve(entry)
    if "seqlens" in data and "max_seqlen" not in shape:
        shape = {**shape, "max_seqlen": int(np.max(data["seqlens"], initial=0))}
    dtypes = {t.name: t.dtype for t in problem.inputs}
    tens = {name: to_torch(arr, dtypes[name], device) for name, arr in data.items()}
    outs: dict[str, torch.Tensor] = {}
    for t in problem.outputs:
        dims = kinp.dims(t, shape)
        buf = torch.empty(dims, dtype=_TORCH[t.dtype], device=device)
        if nan_fill:
            buf.view(torch.uint8).fill_(NAN_BYTE)
        outs[t.name] = buf
    if launched is None:
        got = fn(tens, shape, outs)
        torch.cuda.synchronize()
    else:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
            got = fn(tens, shape, outs)
            torch.cuda.synchronize()
        launched.extend(ev.name for ev in prof.events() if ev.device_type.name == "CUDA"
                        and not ev.name.startswith(("Memset", "Memcpy")))
    if raw:
        return got
    return {name: v.to(torch.float64).cpu().numpy() for name, v in got.items()}


def trace_kernels(entry: str, problem: Problem, shape: dict[str, Any],
                  data: dict[str, np.ndarray], timeout_s: float = 600.0) -> list[str]:
    """Names of the GPU kernels one launch of ``entry`` puts on the device, traced in a fresh
    Python process (its first and only CUPTI session), as the reference traces a build in a
    separate nsys job (src/kta/checks/anticheat.py). A process that has opened many profiler
    sessions can stop receiving kernel activity records, which would read as "no kernel"."""
    import json
    import subprocess
    import sys
    import tempfile
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    with tempfile.TemporaryDirectory(prefix="kta_trace_") as d:
        job = Path(d)
        np.savez(job / "inputs.npz", **data)
        (job / "job.json").write_text(json.dumps(
            {"entry": entry, "problem": problem.model_dump(), "shape": shape},
            default=lambda v: v.item() if hasattr(v, "item") else str(v)), encoding="utf-8")
        res = subprocess.run([sys.executable, "-m", "kta_b200.runners", "--trace", str(job)],
                             cwd=root, capture_output=True, text=True, timeout=timeout_s)
        if res.returncode != 0:
            raise RuntimeError(f"kernel trace of {entry} failed:\n{res.stderr[-2000:]}")
        return list(json.loads((job / "kernels.json").read_text(encoding="utf-8")))


def _trace_main(job_dir: str) -> None:
    import json
    from pathlib import Path

    job = Path(job_dir)
    spec = json.loads((job / "job.json").read_text(encoding="utf-8"))
    with np.load(job / "inputs.npz") as z:
        data = {k: z[k] for k in z.files}
    names: list[str] = []
    run(spec["entry"], Problem.model_validate(spec["problem"]), spec["shape"], data,
        nan_fill=True, raw=True, launched=names)
    (job / "kernels.json").write_text(json.dumps(names), encoding="utf-8")


if __name__ == "__main__":
    import sys

    if len(sys.argv) == 3 and sys.argv[1] == "--trace":
        _trace_main(sys.argv[2])
    else:
        raise SystemExit("usage: python -m kta_b200.runners --trace <job dir>")
