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
