"""The device watchdog that bounds every wait of the library's kernels, exercised on the GPU
without a fault: kta_watchdog_selftest waits for a barrier phase that nothing completes, the
bounded wait expires, records KTA_ERR_DEVICE_TIMEOUT and its site in the device status block
and the kernel returns. The host reads the status, and the context stays usable (a GEMM run
afterwards is correct and leaves the status clean)."""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SELFTEST_SITE = 0x7F01
TIMEOUT = 5  # KTA_ERR_DEVICE_TIMEOUT


def test_bounded_wait_expires_and_reports(cuda_device):
    from kta_b200 import lib

    L = lib.load()
    lib.device_status(clear=True)
    t0 = time.perf_counter()
    assert L.kta_watchdog_selftest(20_000_000, None) == 0  # 20 ms
    status = lib.device_status(clear=True)
    elapsed = time.perf_counter() - t0
    assert status[0] == TIMEOUT and status[1] == SELFTEST_SITE and status[3] >= 1, status
    assert 0.015 < elapsed < 5.0, elapsed  # it waited about its limit, then returned
    assert lib.device_status(clear=True)[0] == 0


def test_context_usable_after_the_watchdog_fired(cuda_device):
    from kta_b200 import lib, ops

    L = lib.load()
    assert L.kta_watchdog_selftest(2_000_000, None) == 0
    assert lib.device_status(clear=True)[0] == TIMEOUT
    g = torch.Generator().manual_seed(5)
    a = torch.randn(256, 512, generator=g).to(torch.bfloat16)
    b = torch.randn(384, 512, generator=g).to(torch.bfloat16)
    c = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    ref = a.double().numpy() @ b.double().numpy().T
    assert np.allclose(c.double().cpu().numpy(), ref, rtol=1e-2, atol=1e-1)
    assert lib.device_status(clear=True)[0] == 0
