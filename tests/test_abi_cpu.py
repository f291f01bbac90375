"""The drop-in boundary on CPU: both C-ABI libraries load without a GPU and
export every symbol their public headers declare (include/opworks_llama.h,
include/opworks_ops.h), including the 11 symbols of the reference's
src/llama_c_api.cu:54-159; and calls that fail before touching the device
follow the reference's error convention (NULL/-1 plus a message)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBS = {
    "opworks_llama.h": os.path.join(ROOT, "opworks_b200", "lib", "libopworks_llama.so"),
    "opworks_ops.h": os.path.join(ROOT, "opworks_b200", "lib", "libopworks_ops.so"),
}
REFERENCE_SYMBOLS = [
    "opw_llama_load", "opw_llama_free", "opw_llama_create_session", "opw_llama_destroy_session",
    "opw_llama_reset_session", "opw_llama_prefill", "opw_llama_decode_step", "opw_llama_is_eos",
    "opw_llama_last_logits", "opw_llama_vocab_size", "opw_llama_last_error",
]


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"OPW_API\s+[\w\s\*]+?\b(opw_\w+)\s*\(", text)))


def load(path):
    if not os.path.exists(path):
        pytest.skip(f"{path} not built")
    return ctypes.CDLL(path)


@pytest.mark.parametrize("header", sorted(LIBS))
def test_every_declared_symbol_is_exported(header):
    names = declared(header)
    assert len(names) >= (20 if header == "opworks_ops.h" else 11)
    lib = load(LIBS[header])
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_reference_symbols_declared_and_exported():
    names = declared("opworks_llama.h")
    for sym in REFERENCE_SYMBOLS:
        assert sym in names
    lib = load(LIBS["opworks_llama.h"])
    for sym in REFERENCE_SYMBOLS:
        assert hasattr(lib, sym)


def test_internal_symbols_are_hidden():
    # kernels and C++ helpers stay local to each library, so two libraries
    # (ours and the reference's) can share a process
    out = os.popen(f"nm -D --defined-only {LIBS['opworks_llama.h']}").read()
    exported = [line.split()[-1] for line in out.splitlines() if " T " in line]
    assert exported and all(name.startswith("opw_") for name in exported), exported[:10]


def test_load_error_convention_without_device_work():
    lib = load(LIBS["opworks_llama.h"])
    lib.opw_llama_load.restype = ctypes.c_void_p
    lib.opw_llama_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_last_error.restype = ctypes.c_char_p
    err = ctypes.create_string_buffer(64)
    h = lib.opw_llama_load(b"/nonexistent/model.pack", err, 64)
    assert not h
    assert err.value  # message, NUL-terminated within err_len
    assert len(err.value) <= 63
    assert lib.opw_llama_last_error()
