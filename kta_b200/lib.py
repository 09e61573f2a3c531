"""ctypes binding of libkta_b200.so, the C ABI declared in include/kta_b200.h.

The library is loaded from this package directory (built in-tree by ``kta_b200.build``).
There is no fallback: if the library is missing or lacks a symbol, ``load()`` raises
``KtaLibraryError``; a nonzero status from an entry raises ``KtaError``.

Argument conventions follow the reference's `so` launcher (src/kta/measure/bench.py:80-98):
device addresses as unsigned 64-bit integers, sizes as 64-bit integers, a CUDA stream handle
(``torch.cuda.current_stream().cuda_stream``) or 0 for the legacy default stream.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkta_b200.so"

KTA_OK = 0
STATUS_NAMES = {
    0: "KTA_OK",
    1: "KTA_ERR_INVALID_ARG",
    2: "KTA_ERR_UNSUPPORTED",
    3: "KTA_ERR_ALIGN",
    4: "KTA_ERR_LAUNCH",
    5: "KTA_ERR_DEVICE_TIMEOUT",
    6: "KTA_ERR_NO_DEVICE",
    7: "KTA_ERR_WORKSPACE",
    8: "KTA_ERR_CUDA",
    9: "KTA_ERR_DEVICE_BOUNDS",
}

_u64, _i64, _i32, _u32 = ctypes.c_uint64, ctypes.c_int64, ctypes.c_int32, ctypes.c_uint32
_f32, _ptr, _size = ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes); every symbol include/kta_b200.h declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "kta_abi_version": (ctypes.c_int, []),
    "kta_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "kta_device_status": (ctypes.c_int, [ctypes.POINTER(_u32), ctypes.c_int]),
    "kta_sm_count": (ctypes.c_int, []),
    "kta_watchdog_selftest": (ctypes.c_int, [_u64, _ptr]),
    "kta_last_error": (ctypes.c_int, []),
    "kta_gemm_bf16": (ctypes.c_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _ptr]),
    "kta_gemm_f16": (ctypes.c_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _ptr]),
    "kta_gemm_nn_bf16": (
        ctypes.c_int,
        [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _ptr],
    ),
    "kta_gemm_nn_f16": (
        ctypes.c_int,
        [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _ptr],
    ),
    "kta_gemm_fp8_blockscaled": (
        ctypes.c_int,
        [_ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr],
    ),
    "kta_attn_fwd_causal_bf16": (
        ctypes.c_int,
        [_ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _f32, _ptr],
    ),
    "kta_decode_workspace_bytes": (_size, [_i64, _i64, _i64, _i64, _i64]),
    "kta_decode_gqa_bf16": (
        ctypes.c_int,
        [_ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _ptr, _size,
         _ptr],
    ),
    "kta_decode_gqa_bf16_noalloc": (
        ctypes.c_int,
        [_ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _ptr],
    ),
    "kta_gemm_w4a16_f16": (ctypes.c_int,
                           [_ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _ptr]),
    "kta_gemm_nvfp4_f16": (ctypes.c_int, [_ptr, _ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr]),
    "kta_so_w4gemm_f16": (None, [_u64, _u64, _u64, _u64, _i32, _i32, _i32]),
    "kta_so_nvfp4gemm_f16": (None, [_u64, _u64, _u64, _u64, _i32, _i32, _i32]),
    "kta_moe_gemm_f16": (ctypes.c_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _ptr]),
    "kta_moe_gemm_bf16": (ctypes.c_int, [_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _ptr]),
    "kta_so_moe_gemm_f16": (None, [_u64, _u64, _u64, _i32, _i32, _i32, _i32]),
    "kta_rmsnorm_f16": (ctypes.c_int, [_ptr, _ptr, _ptr, _i64, _i64, _f32, _ptr]),
    "kta_rmsnorm_bf16": (ctypes.c_int, [_ptr, _ptr, _ptr, _i64, _i64, _f32, _ptr]),
    "kta_softmax_f16": (ctypes.c_int, [_ptr, _ptr, _i64, _i64, _ptr]),
    "kta_softmax_bf16": (ctypes.c_int, [_ptr, _ptr, _i64, _i64, _ptr]),
    "kta_so_rmsnorm_f16": (None, [_u64, _u64, _u64, _i32, _i32]),
    "kta_so_softmax_f16": (None, [_u64, _u64, _i32, _i32]),
    "kta_so_gemm_bf16": (None, [_u64, _u64, _u64, _i32, _i32, _i32]),
    "kta_so_gemm_f16": (None, [_u64, _u64, _u64, _i32, _i32, _i32]),
    "kta_so_gemm_nn_f16": (None, [_u64, _u64, _u64, _i32, _i32, _i32]),
    "kta_so_gemm_nn_bf16": (None, [_u64, _u64, _u64, _i32, _i32, _i32]),
}


class KtaLibraryError(RuntimeError):
    """libkta_b200.so is missing, unloadable or lacks a declared symbol."""


class KtaError(RuntimeError):
    """A libkta_b200 entry returned a nonzero kta_status code."""

    def __init__(self, entry: str, status: int, text: str) -> None:
        super().__init__(f"{entry}: {STATUS_NAMES.get(status, status)} ({text})")
        self.entry = entry
        self.status = status


_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


def load(path: Path | None = None) -> ctypes.CDLL:
    """The loaded library with every declared signature set; raises if anything is missing."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise KtaLibraryError(
                f"{p} not found: build it with `python -m kta_b200.build` (no CPU fallback exists)"
            )
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as exc:
            raise KtaLibraryError(f"cannot load {p}: {exc}") from exc
        missing = [name for name in SIGNATURES if not hasattr(lib, name)]
        if missing:
            raise KtaLibraryError(f"{p} lacks declared symbols: {missing}")
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def status_text(status: int) -> str:
    raw = load().kta_status_string(int(status))
    return raw.decode() if raw else str(status)


def check(entry: str, status: int) -> None:
    if status != KTA_OK:
        raise KtaError(entry, int(status), status_text(status))


def call(entry: str, *args: object) -> None:
    """Calls ``entry`` and raises KtaError on a nonzero status."""
    check(entry, getattr(load(), entry)(*args))


def device_status(clear: bool = True) -> list[int]:
    """The device status block (first error code, site, block, failure count), after a
    device synchronisation; cleared when ``clear``."""
    words = (_u32 * 4)()
    check("kta_device_status", load().kta_device_status(words, 1 if clear else 0))
    return [int(w) for w in words]
