"""teenygrad_b200: B200-native (sm_100a) kernels for teenygrad's operator hot path.

The compute lives in ``libteeny_b200.so`` (C ABI: ``include/teeny_b200.h``);
this package is a thin host layer over it.  Importing the package does not
touch the GPU; the first op call loads the library and fails loudly if it is
missing (there is no CPU fallback).
"""
from ._lib import TeenyError, header_functions, lib  # noqa: F401

__all__ = ["TeenyError", "lib", "header_functions", "ops"]


def __getattr__(name):
    if name in ("ops", "decoder"):
        import importlib

        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(name)
