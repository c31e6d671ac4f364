"""Loads libcairn_b200.so (built in-tree by cairn_b200.build) and declares the C ABI of include/cairn_b200.h.

There is no fallback: if the library is missing or fails to load, every call raises CairnError.
"""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libcairn_b200.so"
HEADER = HERE.parent / "include" / "cairn_b200.h"

OK, ERR_SHAPE, ERR_VIEW, ERR_OVERLAP, ERR_OVERFLOW, ERR_CUDA, ERR_TIMEOUT, ERR_ARG, ERR_DEVICE, ERR_SCRATCH = range(10)
BF16, F16, F8E4M3, F8E5M2, TF32 = range(5)
OUT_ACC_F32, OUT_STORE_F32, OUT_BF16 = range(3)
ACT_NONE, ACT_RELU = range(2)


class CairnError(RuntimeError):
    """A guard the reference enforces with cr::trap (an abort) failed, or the device reported an error."""

    def __init__(self, status: int, where: str = ""):
        self.status = status
        text = _status_text(status)
        super().__init__(f"{where}: {text} (status {status})" if where else f"{text} (status {status})")


_z, _p, _i, _f, _u32p, _ip = C.c_size_t, C.c_void_p, C.c_int, C.c_float, C.POINTER(C.c_uint32), C.POINTER(C.c_int)
SIGNATURES: dict[str, tuple] = {
    "cairn_b200_mma_bf16": (_i, [_p, _z, _z, _z, _p, _z, _p, _z, _p, _z]),
    "cairn_b200_mma_f16": (_i, [_p, _z, _z, _z, _p, _z, _p, _z, _p, _z]),
    "cairn_b200_mma_f8e4m3": (_i, [_p, _z, _z, _z, _p, _z, _p, _z, _p, _z]),
    "cairn_b200_mma_f8e5m2": (_i, [_p, _z, _z, _z, _p, _z, _p, _z, _p, _z]),
    "cairn_b200_mma_tf32": (_i, [_p, _z, _z, _z, _p, _z, _p, _z, _p, _z]),
    "cairn_b200_gemm": (_i, [_p, _i, _z, _z, _z, _p, _i, _p, _i, _p, _i, _p, _i]),
    "cairn_b200_gemm_relu_grad": (_i, [_p, _i, _z, _z, _z, _p, _i, _p, _i, _p, _p]),
    "cairn_b200_mse_grad": (_i, [_p, _z, _p, _p, _p, _p]),
    "cairn_b200_saxpy_f32": (_i, [_p, _z, _p, _p, _p, _f]),
    "cairn_b200_sum_f32": (_i, [_p, _z, _p, _p]),
    "cairn_b200_sum_f32_partial": (_i, [_p, _z, _p, _p]),
    "cairn_b200_sum_f32_host": (_i, [_p, _z, _p, C.POINTER(C.c_float)]),
    "cairn_b200_sum_f32_combine": (_i, [_p, _z, C.POINTER(C.c_float)]),
    "cairn_b200_sum_f32_combine_device": (_i, [_p, _p, _z, _p]),
    "cairn_b200_sum_f32_noalloc": (_i, [_p, _z, _p, _p]),
    "cairn_b200_sum_u64": (_i, [_p, _z, _p, _p, _p]),
    "cairn_b200_sum_u64_host": (_i, [_p, _z, _p, C.POINTER(C.c_uint64), _ip]),
    "cairn_b200_stream_status": (_i, [_p]),
    "cairn_b200_watchdog_selftest": (_i, [_p]),
    "cairn_b200_status_string": (C.c_char_p, [_i]),
    "cairn_b200_clock_marks": (_i, [_p, _p, _z]),
    "cairn_b200_sm_count": (_i, []),
    "cairn_b200_version": (_i, []),
}

_lib: C.CDLL | None = None


def header_symbols() -> list[str]:
    """Every entry point include/cairn_b200.h declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(cairn_b200_\w+)\s*\(", text, flags=re.M)))


def lib() -> C.CDLL:
    """The loaded library, with every declared entry typed."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise CairnError(ERR_DEVICE, f"{LIB_PATH.name} is not built (python -m cairn_b200.build)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def _status_text(status: int) -> str:
    try:
        return lib().cairn_b200_status_string(status).decode()
    except Exception:  # the library itself may be what failed to load
        return "libcairn_b200.so unavailable"


def check(status: int, where: str = "") -> None:
    if status != OK:
        raise CairnError(status, where)
