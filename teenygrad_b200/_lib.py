"""ctypes binding of libteeny_b200.so (the C ABI declared in include/teeny_b200.h).

The library is loaded from this package directory only.  There is no CPU or
PyTorch fallback: if the shared object is missing or the device is not an
sm_100 GPU, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libteeny_b200.so")
HEADER = os.path.join(HERE, "..", "include", "teeny_b200.h")

TB_OK, TB_ERR_ARG, TB_ERR_SHAPE, TB_ERR_ALIGN, TB_ERR_CUDA = 0, 1, 2, 3, 4
TB_ERR_UNSUPPORTED, TB_ERR_DEVICE, TB_ERR_NCCL, TB_ERR_OOM = 5, 6, 7, 8
TB_F32, TB_BF16, TB_I8, TB_I32 = 0, 1, 2, 3
TB_ACT = {"silu": 0, "gelu_tanh": 1, "relu": 2, "sigmoid": 3}
TB_EPI_BIAS, TB_EPI_RESIDUAL, TB_EPI_SWIGLU, TB_EPI_OUT_F32 = 1, 2, 4, 8


class TeenyError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


_lib = None
_lock = threading.Lock()


def header_functions() -> list[str]:
    """Names of every entry point declared in include/teeny_b200.h."""
    text = open(HEADER).read()
    return re.findall(r"^TB_API\s+[\w\s\*]+?\b(tb_\w+)\s*\(", text, flags=re.M)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise TeenyError(TB_ERR_UNSUPPORTED,
                                     f"{LIB_PATH} is missing: run teenygrad_b200/build.py "
                                     "(there is no CPU fallback)")
                l = ctypes.CDLL(LIB_PATH)
                l.tb_strerror.restype = ctypes.c_char_p
                l.tb_last_error.restype = ctypes.c_char_p
                l.tb_last_error.argtypes = [ctypes.c_void_p]
                _lib = l
    return _lib


def strerror(status: int) -> str:
    return lib().tb_strerror(ctypes.c_int(status)).decode()


def check(ctx_ptr, status: int) -> None:
    if status != TB_OK:
        detail = lib().tb_last_error(ctx_ptr).decode() if ctx_ptr else ""
        raise TeenyError(status, f"{strerror(status)}: {detail}")
