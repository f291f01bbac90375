"""OpWorks-B200: B200-native (sm_100a) rebuild of the OpWorks Llama hot path.

The product is two in-tree shared libraries with C ABIs:

* ``opworks_b200/lib/libopworks_ops.so``   — operator layer (``include/opworks_ops.h``)
* ``opworks_b200/lib/libopworks_llama.so`` — Llama runtime (``include/opworks_llama.h``)

This package only locates and binds them (ctypes). There is no fallback: if a
library is missing, loading raises, so a GPU run can never silently take a
CPU or library path.
"""

from __future__ import annotations

import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "opworks_b200", "lib")

_libs = {}


def lib_path(name):
    return os.path.join(LIBDIR, name)


def load(name):
    """dlopen an in-tree library (raises if it has not been built)."""
    if name not in _libs:
        path = lib_path(name)
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with `python -m opworks_b200.build` "
                               "(the CUDA path has no fallback)")
        _libs[name] = ctypes.CDLL(path)
    return _libs[name]


def ops_lib():
    from . import ops

    return ops.bind(load("libopworks_ops.so"))


def llama_lib():
    from . import llama

    return llama.bind(load("libopworks_llama.so"))
