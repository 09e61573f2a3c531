"""Plug-in runners with a planted fault, for the checker self-test
(tests/test_checker_selftest_gpu.py). Each wraps a correct libkta_b200 launch and plants one
mistake the checker must catch, the way src/kta/checks/selftest.py:35-59 builds deliberately
broken modules. No fault touches the GPU: the mistakes are made on the host (a copy) or by a
correct kernel. The checker reaches these through ``kta_b200.runners.resolve`` as
``"tests.planted_runners:<name>"`` (also in the fresh process that traces kernels).
"""

from __future__ import annotations

import torch

from kta_b200 import ops

_calls = {"n": 0}


def gemm_row_dropped(t, shape, out):
    """A correct GEMM whose row 3 of C is then overwritten with NaN from the host (a copy, no
    kernel): an unwritten row, as a kernel that skips it leaves the NaN fill."""
    c = ops.gemm(t["A"], t["B"], out=out["C"])
    row = torch.full((c.shape[1],), float("nan"), dtype=c.dtype)
    c[min(3, c.shape[0] - 1)].copy_(row)
    return {"C": c}


def fp8_scale_doubled(t, shape, out):
    """The FP8 kernel launched with the first weight block's scale doubled (changed on the
    host, copied back): a wrong scale, as a kernel that reads the wrong block would apply."""
    sb = t["sb"].cpu()
    sb[0, 0] *= 2.0
    sb = sb.to(t["sb"].device)
    return {"C": ops.gemm_fp8_blockscaled(t["A"], t["sa"], t["B"], sb, out=out["C"])}


def gemm_with_foreign_kernel(t, shape, out):
    """A correct GEMM that also launches a torch kernel: a launch the library did not
    declare, as a module that calls a vendor library would."""
    c = ops.gemm(t["A"], t["B"], out=out["C"])
    torch.ones(8, device=c.device).mul_(2.0)
    return {"C": c}


def gemm_not_deterministic(t, shape, out):
    """A GEMM whose every second call differs in one element (changed from the host): a
    repeat of the same inputs that does not give the same bytes."""
    c = ops.gemm(t["A"], t["B"], out=out["C"])
    _calls["n"] += 1
    if _calls["n"] % 2 == 0:
        v = c[0, :1].cpu().float() + 1.0
        c[0, :1].copy_(v.to(c.dtype))
    return {"C": c}
