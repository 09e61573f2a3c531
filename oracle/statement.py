"""The reference's statement runner, on the CPU.

src/kta/checks/scripts/ref_torch.py:17-45 executes ``Problem.reference_impl`` with the input
tensors and the shape variables in scope, once widened to FP64 (the reference) and, with
``library``, once in the inputs' own dtype (the "library" result the verdict compares
against). It runs there on "cuda"; here the same two executions run on the host cores with
torch (the reference's CPU path, also the timed CPU baseline of bench.py).
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch


def run_f64(statement: str, inputs: dict[str, torch.Tensor], shape: dict[str, Any],
            outputs: list[str]) -> dict[str, np.ndarray]:
    """``statement`` on the inputs widened to float64 (ref_torch.py:28-38, device cpu)."""
    scope: dict[str, Any] = {"torch": torch, **shape}
    for name, t in inputs.items():
        if t.dtype in (torch.int32, torch.int64):
            scope[name] = t.clone()
        else:
            scope[name] = t.to(torch.float64)
    exec(statement, scope)  # noqa: S102 - the case's own statement, as the reference runs it
    return {name: scope[name].to(torch.float64).numpy() for name in outputs}


def run_library(statement: str, inputs: dict[str, torch.Tensor], shape: dict[str, Any],
                outputs: list[str] | None = None) -> dict[str, torch.Tensor]:
    """``statement`` on the inputs in their own dtype (ref_torch.py:39-43, device cpu)."""
    scope: dict[str, Any] = {"torch": torch, **shape, **inputs}
    exec(statement, scope)  # noqa: S102
    names = outputs if outputs is not None else [n for n in ("C", "O", "LSE") if n in scope]
    return {name: scope[name] for name in names}
