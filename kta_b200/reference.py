"""The case's reference outputs, computed on the GPU (the product checker's reference).

Mirrors src/kta/checks/reference.py:55-117 and src/kta/checks/scripts/ref_torch.py:17-45:
``Problem.reference_impl`` is a Python statement over torch tensors named like the Problem's
inputs and outputs, with the shape variables in scope; it runs on the exact input bytes
widened to FP64 (or FP32 when asked), and with ``library`` once more in the inputs' own dtype
(reduced-precision reductions off) — the "library" result the verdict compares against.
Integer inputs stay integers. Outputs come back as float64 numpy arrays.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from kta_b200 import inputs as kinp
from kta_b200.schemas import Problem

_TORCH_OF = {
    "f16": torch.float16, "float16": torch.float16, "bf16": torch.bfloat16,
    "bfloat16": torch.bfloat16, "f32": torch.float32, "float32": torch.float32,
    "f64": torch.float64, "float64": torch.float64, "i32": torch.int32, "int32": torch.int32,
    "i64": torch.int64, "int64": torch.int64, "e4m3": torch.float8_e4m3fn,
}


class NotSupported(ValueError):
    pass


def to_torch(arr: np.ndarray, dtype: str, device: str | torch.device) -> torch.Tensor:
    """Host bytes of a case tensor (bf16 / e4m3 as bit patterns) as a torch tensor."""
    a = np.ascontiguousarray(arr)
    if dtype in ("bf16", "bfloat16"):
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    if dtype == "e4m3":
        return torch.from_numpy(a.view(np.uint8)).view(torch.float8_e4m3fn).to(device)
    return torch.from_numpy(a).to(device)


@dataclass(frozen=True)
class Reference:
    outputs: list[dict[str, np.ndarray]]            # per input set, FP64
    compute: str
    library: list[dict[str, np.ndarray]] | None = None


def reference(problem: Problem, shape: dict[str, Any], sets: list[dict[str, np.ndarray]],
              compute: str = "f64", library: bool = False,
              device: str | torch.device = "cuda") -> Reference:
    if problem.reference_impl.startswith("none"):
        raise NotSupported(f"problem {problem.name} has no reference: {problem.reference_impl}")
    cdt = {"f64": torch.float64, "f32": torch.float32}[compute]
    dtypes = {t.name: t.dtype for t in problem.inputs}
    outs: list[dict[str, np.ndarray]] = []
    libs: list[dict[str, np.ndarray]] | None = [] if library else None
    prev16 = torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction
    prevbf = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
    try:
        if library:
            torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        for data in sets:
            scope: dict[str, Any] = {"torch": torch, **shape}
            low: dict[str, Any] = {"torch": torch, **shape}
            for name, arr in data.items():
                t = to_torch(arr, dtypes[name], device)
                scope[name] = t if not t.dtype.is_floating_point else t.to(cdt)
                if t.dtype == torch.float8_e4m3fn:
                    scope[name] = t.to(torch.float32).to(cdt)
                low[name] = t
            exec(problem.reference_impl, scope)  # noqa: S102 - the case's own statement
            outs.append({t.name: scope[t.name].to(torch.float64).cpu().numpy()
                         for t in problem.outputs})
            if libs is not None:
                exec(problem.reference_impl, low)  # noqa: S102
                libs.append({t.name: low[t.name].to(torch.float64).cpu().numpy()
                             for t in problem.outputs})
    finally:
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = prev16
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = prevbf
    return Reference(outs, compute, libs)


def host_dtype(dtype: str) -> Any:
    return kinp.np_dtype(dtype)
