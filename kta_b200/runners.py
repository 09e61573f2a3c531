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


def run(entry: str, problem: Problem, shape: dict[str, Any], data: dict[str, np.ndarray],
        nan_fill: bool = True, raw: bool = False, device: str = "cuda",
        launched: list[str] | None = None) -> dict[str, Any]:
    """Outputs of one launch as float64 numpy arrays (``raw``: device tensors). With
    ``launched``, the names of the GPU kernels the entry itself launched are appended to it
    (a CUPTI trace through torch.profiler around the launch only; memsets and copies are not
    kernels)."""
    from kta_b200 import inputs as kinp

    if entry not in RUNNERS:
        raise ValueError(f"no runner for entry {entry!r}")
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
        got = RUNNERS[entry](tens, shape, outs)
        torch.cuda.synchronize()
    else:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            got = RUNNERS[entry](tens, shape, outs)
            torch.cuda.synchronize()
        for ev in prof.events():
            if ev.device_type.name == "CUDA" and not ev.name.startswith(("Memset", "Memcpy")):
                launched.append(ev.name)
    if raw:
        return got
    return {name: v.to(torch.float64).cpu().numpy() for name, v in got.items()}
