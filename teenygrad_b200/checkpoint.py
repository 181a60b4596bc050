"""safetensors checkpoints through the library's reader (tb_st_*).

The file is memory-mapped by the library; tensors are read in place.  This
covers teeny-quant's quantised output (utilities/teeny-quant/src/format.rs):
I8 weights with an F32 `<name>_scale` per output channel and a
`quantization_config` metadata entry.  Decoder.load_checkpoint loads a
Llama-layout checkpoint straight into the executor (int8 tensors into the
int8 GEMV layout, not re-quantised).
"""
from __future__ import annotations

import ctypes
import json

import numpy as np

from ._lib import TB_BF16, TB_F32, TB_I8, TB_I32, TeenyError, check, lib

_NP = {TB_F32: np.float32, TB_I8: np.int8, TB_I32: np.int32, TB_BF16: np.uint16}


class SafeTensors:
    """Read-only view of a .safetensors file (needs no GPU)."""

    def __init__(self, path: str):
        self._h = ctypes.c_void_p()
        st = lib().tb_st_open(path.encode(), ctypes.byref(self._h))
        if st != 0:
            raise TeenyError(st, f"tb_st_open({path}) failed")

    def close(self):
        if self._h:
            lib().tb_st_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list[str]:
        l = lib()
        l.tb_st_name.restype = ctypes.c_char_p
        return [l.tb_st_name(self._h, ctypes.c_int(i)).decode() for i in range(l.tb_st_count(self._h))]

    def info(self, name: str):
        """(dtype code or -1, shape, nbytes)."""
        dt, rank = ctypes.c_int(0), ctypes.c_int(8)
        shape = (ctypes.c_int64 * 8)()
        nb = ctypes.c_size_t(0)
        check(None, lib().tb_st_tensor(self._h, name.encode(), ctypes.byref(dt), shape, ctypes.byref(rank), None,
                                       ctypes.byref(nb)))
        return dt.value, tuple(shape[i] for i in range(rank.value)), nb.value

    def numpy(self, name: str) -> np.ndarray:
        """A copy of the tensor (bf16 as uint16 bit patterns)."""
        dt, shape, nb = self.info(name)
        if dt not in _NP:
            raise TeenyError(5, f"{name}: dtype not F32, BF16, I8 or I32")
        ptr = ctypes.c_void_p()
        check(None, lib().tb_st_tensor(self._h, name.encode(), None, None, None, ctypes.byref(ptr), None))
        buf = (ctypes.c_uint8 * nb).from_address(ptr.value)
        return np.frombuffer(buf, dtype=_NP[dt]).reshape(shape).copy()

    def metadata(self, key: str):
        l = lib()
        l.tb_st_metadata.restype = ctypes.c_char_p
        v = l.tb_st_metadata(self._h, key.encode())
        return None if v is None else v.decode()

    def quantization_config(self):
        v = self.metadata("quantization_config")
        return None if v is None else json.loads(v)
