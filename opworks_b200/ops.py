"""ctypes binding of libopworks_ops.so (prototypes of include/opworks_ops.h).

Device pointers are passed as integers (e.g. ``tensor.data_ptr()``); streams as
integers (``torch.cuda.current_stream().cuda_stream``) or 0 for the legacy
default stream. ``check(rc)`` raises ``ValueError`` with the library's message
when an entry point rejected its arguments.
"""

from __future__ import annotations

import ctypes

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float

SIGNATURES = {
    "opw_ops_sync": [P],
    "opw_map_add": [P, P, P, I, P],
    "opw_map_relu": [P, P, I, P],
    "opw_map_scale": [P, P, I, F, P],
    "opw_reduction_workspace_size": [I],
    "opw_reduce": [I, P, P, I, P, I, P],
    "opw_reduce_static": [I, P, P, I, P],
    "opw_softmax": [P, P, I, I, P],
    "opw_layer_norm": [P, P, P, P, I, I, F, P],
    "opw_mat_mul": [P, P, P, I, I, I, I, F, P],
    "opw_matmul_builder": [P, P, P, I, I, I, I, I, P, I, P],
    "opw_rowwise_builder": [I, P, P, P, P, I, I, F, P],
    "opw_rms_norm": [P, P, P, I, I, F, P],
    "opw_linear_f32": [P, P, P, I, I, I, P],
    "opw_linear_bf16": [P, P, P, I, I, I, P],
    "opw_linear_mma_bf16": [P, P, P, I, I, I, P],
    "opw_embedding_f32": [P, P, P, I, I, P],
    "opw_embedding_bf16": [P, P, P, I, I, P],
    "opw_rope": [P, P, I, I, I, I, P],
    "opw_split_heads": [P, P, I, I, I, I, I, P],
    "opw_merge_heads": [P, P, I, I, I, I, I, P],
    "opw_causal_scale": [P, I, I, F, P],
    "opw_swiglu": [P, P, P, I64, P],
    "opw_add": [P, P, P, I64, P],
    "opw_argmax": [P, I, P, P],
    "opw_attention_decode": [P, P, P, P, I, I, I, I, I, P],
    "opw_attention_prefill_chunked": [P, P, P, P, I, I, I, I, I, I, I, P],
    "opw_sample": [P, I, I, P, P, P, P, P],
    "opw_paged_attention_decode": [P, P, P, P, I, P, I, I, I, I, P, P],
    "opw_gemm_bf16x2": [P, P, P, P, I, I, I, I, P],
    "opw_gemm_bf16x2_pair": [P, P, P, P, I, I, I, P],
    "opw_gemm_f16x2": [P, P, P, P, I, I, I, I, P],
    "opw_gemm_f16x2_pair": [P, P, P, P, I, I, I, P],
    "opw_paged_attention_prefill": [P, P, P, P, I, I, I, I, I, I, I, P, I, P],
}


class OpsLib:
    def __init__(self, lib):
        self.lib = lib
        lib.opw_ops_last_error.restype = ctypes.c_char_p
        lib.opw_ops_last_error.argtypes = []
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int

    def last_error(self):
        return self.lib.opw_ops_last_error().decode(errors="replace")

    def check(self, rc):
        if rc != 0:
            raise ValueError(self.last_error())
        return rc

    def __getattr__(self, name):
        fn = getattr(self.lib, "opw_" + name)

        def call(*args):
            return self.check(fn(*[_arg(a) for a in args]))

        return call

    def raw(self, name):
        fn = getattr(self.lib, "opw_" + name)
        return lambda *args: fn(*[_arg(a) for a in args])


def _arg(a):
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a


_cache = {}


def bind(lib):
    key = id(lib)
    if key not in _cache:
        _cache[key] = OpsLib(lib)
    return _cache[key]
