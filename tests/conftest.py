"""Shared pytest configuration: the `gpu` marker and seeded input helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 CUDA device (B200)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip("libkta_b200 needs an sm_100 device")
    from kta_b200 import lib

    lib.load()  # no fallback: a missing or incomplete library fails here
    return torch.device("cuda", 0)
