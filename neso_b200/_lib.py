"""ctypes binding of ``libneso_b200.so`` (the C ABI declared in include/neso_b200.h).

The library is loaded from this package directory only. There is no fallback:
if the shared object is missing or fails to load, :func:`lib` raises
:class:`NesoLibraryError`, so no caller can silently run a CPU path.
"""
from __future__ import annotations

import ctypes
import os
import re
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libneso_b200.so"
HEADER_PATH = _PKG.parent / "include" / "neso_b200.h"

NESO_OK = 0
NESO_ERR_INVALID_ARG = -1
NESO_ERR_MISALIGNED = -2
NESO_ERR_UNSUPPORTED = -3
NESO_ERR_GRID = -4
NESO_ERR_LAUNCH = -5
NESO_ERR_DEVICE_TIMEOUT = -6
NESO_ERR_NO_DEVICE = -7

_CODE_NAMES = {
    NESO_OK: "NESO_OK",
    NESO_ERR_INVALID_ARG: "NESO_ERR_INVALID_ARG",
    NESO_ERR_MISALIGNED: "NESO_ERR_MISALIGNED",
    NESO_ERR_UNSUPPORTED: "NESO_ERR_UNSUPPORTED",
    NESO_ERR_GRID: "NESO_ERR_GRID",
    NESO_ERR_LAUNCH: "NESO_ERR_LAUNCH",
    NESO_ERR_DEVICE_TIMEOUT: "NESO_ERR_DEVICE_TIMEOUT",
    NESO_ERR_NO_DEVICE: "NESO_ERR_NO_DEVICE",
}


class NesoLibraryError(RuntimeError):
    """The native library is missing or could not be loaded."""


class NesoError(RuntimeError):
    """A C-ABI call returned a non-zero status (mirrors the reference's
    RuntimeError on a failed Metal dispatch, src/neso/backend/driver.py:314-317)."""

    def __init__(self, code: int, message: str, func: str = ""):
        self.code = code
        self.func = func
        super().__init__(f"{func}: {_CODE_NAMES.get(code, code)}: {message}")


_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_u32 = ctypes.c_uint32
_f32 = ctypes.c_float
_int = ctypes.c_int
_ip = ctypes.POINTER(ctypes.c_int)
_GRID = [_u32, _u32, _u32]

# name -> (restype, argtypes); kept in the order of include/neso_b200.h
SIGNATURES: dict[str, tuple[object, list]] = {
    "neso_last_error_string": (ctypes.c_char_p, []),
    "neso_version": (_int, []),
    "neso_set_device": (_int, [_int]),
    "neso_device_status": (_int, [_int, _ip, _ip, _ip, _ip]),
    "neso_clear_device_status": (_int, [_int]),
    "neso_selftest_wait_timeout": (_int, [_int, _p]),
    "neso_kernel_metadata": (ctypes.c_char_p, [ctypes.c_char_p]),
    "neso_vector_add": (_int, [_p, _p, _p, _i32, _i32, *_GRID, _p]),
    "neso_add_kernel": (_int, [_p, _p, _p, _i32, _i32, *_GRID, _p]),
    "neso_scale": (_int, [_p, _p, _f32, _i32, _i32, *_GRID, _p]),
    "neso_rmsnorm_kernel": (_int, [_p, _p, _p, _i32, _i32, _f32, _i32, *_GRID, _p]),
    "neso_residual_rmsnorm_kernel": (_int, [_p, _p, _p, _p, _i32, _i32, _f32, _i32, *_GRID, _p]),
    "neso_rope_kernel": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, *_GRID, _p]),
    "neso_silu_kernel": (_int, [_p, _p, _i32, _i32, *_GRID, _p]),
    "neso_softmax_kernel": (_int, [_p, _p, _i32, _i32, _i32, _i32, *_GRID, _p]),
    "neso_per_channel_dequant_kernel": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _i32, *_GRID, _p]),
    "neso_grouped_dequant_kernel": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, *_GRID, _p]),
    "neso_quantize_kernel": (_int, [_p, _p, _p, _i32, _i32, *_GRID, _p]),
    "neso_flash_attention_fwd": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _f32, _i32, *_GRID, _p]),
    "neso_rel_pos_fa2_fwd": (_int, [_p, _p, _p, _p, _p, _i32, _i32, _f32, _i32, _i32, _i32, *_GRID, _p]),
    "neso_flash_attention_fwd_msl": (_int, [_p, _p, _p, _p, _i32, _i32, _f32] + [_i32] * 5 + [*_GRID, _p]),
    "neso_flash_attention_opt": (_int, [_p, _p, _p, _p, _i32, _i32, _f32] + [_i32] * 5 + [*_GRID, _p]),
    "neso_flash_attention_d128": (_int, [_p, _p, _p, _p, _i32, _i32, _f32] + [_i32] * 5 + [*_GRID, _p]),
    "neso_fa2_fwd": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _i32, _f32, _i32, _p]),
    "neso_fa2_fwd_relpos_table": (_int, [_p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _f32, _i32, _p]),
    "neso_matmul_kernel": (_int, [_p, _p, _p] + [_i32] * 12 + [*_GRID, _p]),
    "neso_matmul_tiled": (_int, [_p, _p, _p] + [_i32] * 6 + [*_GRID, _p]),
    "neso_w8a16_matmul": (_int, [_p, _p, _p] + [_i32] * 7 + [*_GRID, _p]),
    "neso_w8a16_scaled_matmul": (_int, [_p, _p, _p, _p] + [_i32] * 7 + [*_GRID, _p]),
    "neso_w8a16_matmul_kernel": (_int, [_p, _p, _p, _p] + [_i32] * 12 + [*_GRID, _p]),
    "neso_w8a16_matmul_kernel_i32": (_int, [_p, _p, _p, _p] + [_i32] * 12 + [*_GRID, _p]),
    "neso_w8a16_matmul_mnk": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _p]),
    "neso_w4a16_g128_matmul": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _p]),
    "neso_w8a16_matmul_mnk_noalloc": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _p]),
}

_lib: ctypes.CDLL | None = None


def header_functions() -> list[str]:
    """Names of every function declared in include/neso_b200.h."""
    text = HEADER_PATH.read_text()
    return re.findall(r"^\s*(?:NESO_API\s+)?(?:const\s+)?\w+\*?\s+(neso_\w+)\s*\(", text, flags=re.M)


def lib() -> ctypes.CDLL:
    """Load the native library (once). Raises NesoLibraryError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise NesoLibraryError(
            f"{LIB_PATH} is missing: build it with `python -m neso_b200.build` "
            "(there is no CPU fallback)")
    try:
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_LOCAL | getattr(os, "RTLD_NOW", 2))
    except OSError as e:
        raise NesoLibraryError(f"failed to load {LIB_PATH}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


def last_error() -> str:
    msg = lib().neso_last_error_string()
    return msg.decode() if msg else ""


def check(rc: int, func: str = "") -> None:
    if rc != NESO_OK:
        raise NesoError(rc, last_error(), func)


def call(name: str, *args) -> None:
    """Call a C-ABI entry point and raise NesoError on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    check(rc, name)
