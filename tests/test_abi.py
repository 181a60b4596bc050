"""The C-ABI library loads without a GPU and exports every declared entry point."""
import ctypes
import os
import re

import pytest

import teenygrad_b200 as tg
from teenygrad_b200 import _lib


def test_library_exports_every_header_symbol():
    names = tg.header_functions()
    assert len(names) >= 20
    l = tg.lib()
    missing = [n for n in names if not hasattr(l, n)]
    assert not missing, missing


def test_header_is_plain_c():
    text = open(_lib.HEADER).read()
    # no C++ or torch types across the boundary
    for bad in ("std::", "torch", "at::", "template", "namespace", "class "):
        assert bad not in text
    assert 'extern "C"' in text


def test_strerror_and_version_need_no_gpu():
    l = tg.lib()
    assert l.tb_abi_version() == 1
    assert _lib.strerror(0) == "ok"
    assert "shape" in _lib.strerror(2)


def test_init_without_sm100_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    ctx = ctypes.c_void_p()
    st = tg.lib().tb_init(ctypes.byref(ctx), 0)
    assert st != 0 and not ctx.value


def test_ops_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from teenygrad_b200 import ops
    with pytest.raises(tg.TeenyError):
        ops.rms_norm(torch.ones(4, 8), torch.ones(8))


def test_no_oracle_import_in_product():
    root = os.path.dirname(_lib.HERE)
    for dirpath, _, files in os.walk(_lib.HERE):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"^\s*(import|from)\s+oracle", src, flags=re.M), f
                assert "liboracle" not in src, f


def test_output_row_stride_and_workspace_need_no_gpu():
    l = tg.lib()
    out = ctypes.c_int64(0)
    # linear rows padded to 16 bytes (LinearForward::forward_output_row_stride)
    for dt, n, want in ((0, 6, 8), (0, 48, 48), (1, 6, 8), (1, 24, 24), (1, 25, 32)):
        assert l.tb_output_row_stride(0, dt, ctypes.c_int64(n), ctypes.byref(out)) == 0
        assert out.value == want, (dt, n, out.value)
    assert l.tb_output_row_stride(1, 0, ctypes.c_int64(6), ctypes.byref(out)) == 0 and out.value == 6   # matmul: dense
    assert l.tb_output_row_stride(99, 0, ctypes.c_int64(6), ctypes.byref(out)) != 0
    b = ctypes.c_size_t(123)
    shape = (ctypes.c_int64 * 9)(32, 64, 64, 56, 56, 3, 3, 1, 1)
    assert l.tb_workspace_bytes(7, 1, shape, 9, ctypes.byref(b)) == 0 and b.value > 32 * 56 * 56 * 64 * 2
    assert l.tb_workspace_bytes(7, 0, shape, 9, ctypes.byref(b)) == 0 and b.value == 0   # f32 conv: none
    assert l.tb_workspace_bytes(0, 1, None, 0, ctypes.byref(b)) == 0 and b.value == 0    # linear: none
