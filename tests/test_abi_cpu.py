"""The C ABI without a GPU: the library loads, exports exactly what include/kta_b200.h
declares, and rejects bad arguments with the documented status codes before any device
work. No compute call is made here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from kta_b200 import lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kta_b200.h"
NO_GPU = not torch.cuda.is_available()


def declared() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|void|size_t|const char\*)\s+(kta_\w+)\(", text,
                                 re.M)))


def test_header_declarations_are_all_exported_and_bound():
    names = declared()
    assert len(names) >= 15
    so = ctypes.CDLL(str(lib.LIB_PATH))
    for n in names:
        assert hasattr(so, n), n
    assert sorted(lib.SIGNATURES) == names


def test_version_and_status_text():
    L = lib.load()
    assert L.kta_abi_version() == 1
    for code, name in lib.STATUS_NAMES.items():
        assert lib.status_text(code) and isinstance(lib.status_text(code), str), name
    assert lib.status_text(77) == "unknown status"


ALIGNED = 0x10000
MISALIGNED = 0x10002


@pytest.mark.parametrize("entry", ["kta_gemm_bf16", "kta_gemm_f16", "kta_gemm_nn_bf16",
                                   "kta_gemm_nn_f16"])
def test_gemm_argument_checks(entry):
    f = getattr(lib.load(), entry)
    assert f(None, ALIGNED, ALIGNED, 64, 64, 64, 64, 64, 64, None) == 1
    assert f(ALIGNED, ALIGNED, ALIGNED, 0, 64, 64, 64, 64, 64, None) == 1
    assert f(ALIGNED, ALIGNED, ALIGNED, 64, 64, 64, 32, 64, 64, None) == 1  # lda < K
    assert f(MISALIGNED, ALIGNED, ALIGNED, 64, 64, 64, 64, 64, 64, None) == 3
    assert f(ALIGNED, ALIGNED, ALIGNED, 64, 68, 64, 64, 68, 68, None) in (3,)  # ld not % 8


@pytest.mark.skipif(not NO_GPU, reason="checks the no-device status")
def test_valid_arguments_without_a_device_report_no_device():
    L = lib.load()
    assert L.kta_gemm_bf16(ALIGNED, ALIGNED, ALIGNED, 64, 64, 64, 64, 64, 64, None) == 6
    words = (ctypes.c_uint32 * 4)()
    assert L.kta_device_status(words, 0) == 6


def test_decode_argument_checks():
    L = lib.load()
    ws = L.kta_decode_workspace_bytes(64, 32, 8, 128, 8192)
    assert ws > 0
    assert L.kta_decode_workspace_bytes(64, 32, 8, 64, 8192) == 0  # D != 128
    args = [ALIGNED] * 6
    f = L.kta_decode_gqa_bf16
    assert f(*args, 64, 32, 8, 64, 1000, 8192, 0.1, ALIGNED, ws, None) == 2    # D
    assert f(*args, 64, 32, 1, 128, 1000, 8192, 0.1, ALIGNED, ws, None) == 2   # group 32
    assert f(*args, 64, 32, 8, 128, 1000, 8192, -1.0, ALIGNED, ws, None) == 1  # scale
    assert f(*args, 64, 32, 8, 128, 1000, 8192, 0.1, ALIGNED, ws - 1, None) == 7
    assert f(*args, 64, 32, 8, 128, 1000, 8192, 0.1, None, ws, None) == 7
    assert f(None, *args[1:], 64, 32, 8, 128, 1000, 8192, 0.1, ALIGNED, ws, None) == 1


def test_noalloc_decode_refuses_what_does_not_fit_its_array():
    L = lib.load()
    args = [ALIGNED] * 6
    assert L.kta_decode_gqa_bf16_noalloc(*args, 2048, 1024, 1024, 128, 1024, 64, 0.1,
                                         None) == 2
    assert L.kta_decode_gqa_bf16_noalloc(*args, 0, 32, 8, 128, 1024, 64, 0.1, None) == 1


def test_attention_argument_checks():
    L = lib.load()
    a = [ALIGNED] * 5
    assert L.kta_attn_fwd_causal_bf16(*a, 2, 4, 256, 64, 0.1, None) == 2      # D != 128
    assert L.kta_attn_fwd_causal_bf16(None, *a[1:], 2, 4, 256, 128, 0.1, None) == 1
    assert L.kta_attn_fwd_causal_bf16(*a, 2, 4, 0, 128, 0.1, None) == 1       # S = 0
    assert L.kta_attn_fwd_causal_bf16(*a, 2, 4, 256, 128, 0.0, None) == 1     # scale
    assert L.kta_attn_fwd_causal_bf16(MISALIGNED, *a[1:], 2, 4, 256, 128, 0.1, None) == 3


def test_fp8_argument_checks():
    L = lib.load()
    a = [ALIGNED] * 5
    assert L.kta_gemm_fp8_blockscaled(*a, 128, 128, 100, None) == 3    # K % 16
    assert L.kta_gemm_fp8_blockscaled(*a, 128, 100, 128, None) == 3    # N % 8
    assert L.kta_gemm_fp8_blockscaled(None, *a[1:], 128, 128, 128, None) == 1
    assert L.kta_gemm_fp8_blockscaled(*a, 0, 128, 128, None) == 1


def test_4bit_gemm_argument_checks():
    L = lib.load()
    a = ALIGNED
    w4, nv = L.kta_gemm_w4a16_f16, L.kta_gemm_nvfp4_f16
    assert w4(a, a, a, a, 128, 128, 100, 32, None) == 3     # K % 64
    assert w4(a, a, a, a, 128, 128, 128, 48, None) == 1     # group not a power of two
    assert w4(a, a, a, a, 128, 128, 192, 128, None) == 3    # K % group
    assert w4(a, a, a, a, 128, 100, 128, 32, None) == 3     # N % 8
    assert w4(None, a, a, a, 128, 128, 128, 32, None) == 1
    assert nv(a, a, a, a, 0, 128, 128, None) == 1
    assert nv(a, MISALIGNED, a, a, 128, 128, 128, None) == 3


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_moe_argument_checks(dt):
    f = getattr(lib.load(), f"kta_moe_gemm_{dt}")
    a = ALIGNED
    assert f(a, a, a, 8, 1000, 1024, 2048, None) == 2     # T not a multiple of E
    assert f(a, a, a, 8, 8 * 100, 1024, 2048, None) == 2  # T / E not a multiple of 128
    assert f(a, a, a, 8, 2048, 1020, 2048, None) == 3     # N % 8
    assert f(None, a, a, 8, 2048, 1024, 2048, None) == 1
    assert f(a, a, a, 0, 2048, 1024, 2048, None) == 1
    assert f(a, MISALIGNED, a, 8, 2048, 1024, 2048, None) == 3


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_rowop_argument_checks(dt):
    L = lib.load()
    rms = getattr(L, f"kta_rmsnorm_{dt}")
    smx = getattr(L, f"kta_softmax_{dt}")
    a = ALIGNED
    assert rms(a, a, a, 64, 100, 1e-6, None) == 3        # N % 8
    assert rms(a, a, a, 64, 16392, 1e-6, None) == 2      # N > 16384
    assert rms(a, None, a, 64, 64, 1e-6, None) == 1      # W missing
    assert rms(a, a, a, 0, 64, 1e-6, None) == 1          # M = 0
    assert rms(a, a, a, 64, 64, -1.0, None) == 1         # eps < 0
    assert rms(MISALIGNED, a, a, 64, 64, 1e-6, None) == 3
    assert smx(a, a, 64, 100, None) == 3
    assert smx(None, a, 64, 64, None) == 1
    assert smx(a, MISALIGNED, 64, 64, None) == 3


def test_so_shim_reports_through_last_error():
    L = lib.load()
    L.kta_so_gemm_f16(0, 0, 0, 64, 64, 64)
    assert L.kta_last_error() == 1


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(lib.KtaLibraryError):
        lib.load(tmp_path / "nope.so")


def test_watchdog_selftest_argument_checks():
    L = lib.load()
    assert L.kta_watchdog_selftest(0, None) == 1            # below 1 us
    assert L.kta_watchdog_selftest(20_000_000_000, None) == 1  # above 10 s
