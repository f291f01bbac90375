"""ORACLE — test infrastructure only (parity checker and timed CPU baseline).

ctypes bindings to ``oracle/liboracle.so``, the C++17/OpenMP restatement of the
OpWorks reference math in ``oracle/oracle.cpp``. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm may import this
module; the product (``opworks_b200``, ``include/``) never does.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)


class OrcLlama(ctypes.Structure):
    _fields_ = [
        ("layers", ctypes.c_int), ("hidden", ctypes.c_int), ("inter", ctypes.c_int),
        ("qh", ctypes.c_int), ("kvh", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("vocab", ctypes.c_int), ("eps", ctypes.c_float),
        ("embed", _f32p), ("final_norm", _f32p),
        ("input_norm", ctypes.POINTER(_f32p)), ("q_proj", ctypes.POINTER(_f32p)),
        ("k_proj", ctypes.POINTER(_f32p)), ("v_proj", ctypes.POINTER(_f32p)),
        ("o_proj", ctypes.POINTER(_f32p)), ("post_norm", ctypes.POINTER(_f32p)),
        ("gate_proj", ctypes.POINTER(_f32p)), ("up_proj", ctypes.POINTER(_f32p)),
        ("down_proj", ctypes.POINTER(_f32p)), ("inv_freq", _f32p),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"oracle library missing: {LIB_PATH} (run __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_softmax.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.orc_layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_mat_mul.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_float]
        L.orc_reduce_sum.argtypes = [_f32p, ctypes.c_int64]
        L.orc_reduce_sum.restype = ctypes.c_double
        L.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_linear.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_linear_bf16.argtypes = [_f32p, _u16p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_rope_inv_freq.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_int, ctypes.c_double,
                                        ctypes.c_double, ctypes.c_double, ctypes.c_double, _f32p]
        L.orc_rope.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int]
        L.orc_swiglu.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64]
        L.orc_argmax.argtypes = [_f32p, ctypes.c_int]
        L.orc_argmax.restype = ctypes.c_int
        L.orc_llama_forward.argtypes = [ctypes.POINTER(OrcLlama), _i32p, ctypes.c_int, ctypes.c_int, _f32p, _f32p,
                                        ctypes.c_int, _f32p, _f32p]
        L.orc_llama_decode_batch.argtypes = [ctypes.POINTER(OrcLlama), _i32p, _i32p, ctypes.c_int, _f32p, _f32p,
                                             ctypes.c_int, _f32p]
        L.orc_top_p_sample.argtypes = [_f32p, ctypes.c_int, ctypes.c_double, ctypes.c_double, ctypes.c_double]
        L.orc_top_p_sample.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a, ptype=_f32p):
    return a.ctypes.data_as(ptype)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def softmax(x):
    x = _f32(x)
    out = np.empty_like(x)
    rows, cols = x.shape
    lib().orc_softmax(_p(x), _p(out), rows, cols)
    return out


def layer_norm(x, gamma, beta, eps=1e-5):
    x, gamma, beta = _f32(x), _f32(gamma), _f32(beta)
    out = np.empty_like(x)
    lib().orc_layer_norm(_p(x), _p(out), _p(gamma), _p(beta), x.shape[0], x.shape[1], eps)
    return out


def mat_mul(a, b, epilogue=0, param=0.0):
    a, b = _f32(a), _f32(b)
    M, N = a.shape
    K = b.shape[1]
    out = np.empty((M, K), np.float32)
    lib().orc_mat_mul(_p(a), _p(b), _p(out), M, N, K, epilogue, param)
    return out


def reduce_sum(x):
    x = _f32(x).ravel()
    return lib().orc_reduce_sum(_p(x), x.size)


def rms_norm(x, w, eps):
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(w), _p(out), x.shape[0], x.shape[1], eps)
    return out


def linear(x, w):
    x, w = _f32(x), _f32(w)
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    lib().orc_linear(_p(x), _p(w), _p(out), x.shape[0], x.shape[1], w.shape[0])
    return out


def linear_bf16(x, w_bits):
    x = _f32(x)
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    out = np.empty((x.shape[0], w_bits.shape[0]), np.float32)
    lib().orc_linear_bf16(_p(x), _p(w_bits, _u16p), _p(out), x.shape[0], x.shape[1], w_bits.shape[0])
    return out


def rope_inv_freq(head_dim, theta, scaling=None):
    out = np.empty(head_dim // 2, np.float32)
    if scaling:
        lib().orc_rope_inv_freq(head_dim, theta, 1, scaling["factor"], scaling["low_freq_factor"],
                                scaling["high_freq_factor"], scaling["original_max_position_embeddings"], _p(out))
    else:
        lib().orc_rope_inv_freq(head_dim, theta, 0, 1.0, 1.0, 1.0, 1.0, _p(out))
    return out


def rope(x, inv_freq, heads, head_dim, pos_start):
    x = _f32(x).copy()
    inv_freq = _f32(inv_freq)
    lib().orc_rope(_p(x), _p(inv_freq), x.shape[0], heads, head_dim, pos_start)
    return x


def attention(q, k, v):
    """q [T, qh, D], k/v [S, kvh, D] -> [T, qh, D] (causal, queries at the end)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    T, qh, D = q.shape
    S, kvh, _ = k.shape
    out = np.empty_like(q)
    lib().orc_attention(_p(q), _p(k), _p(v), _p(out), T, S, qh, kvh, D)
    return out


def swiglu(g, u):
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), _p(out), g.size)
    return out


def argmax(x):
    x = _f32(x).ravel()
    return int(lib().orc_argmax(_p(x), x.size))


def top_p_sample(logits, temperature, top_p, u):
    logits = _f32(logits).ravel()
    return int(lib().orc_top_p_sample(_p(logits), logits.size, float(temperature), float(top_p), float(u)))


class Llama:
    """CPU Llama over host fp32 weights (dict name -> array, HF names)."""

    def __init__(self, cfg, weights):
        self.cfg = cfg
        c = cfg
        self.L = c["num_hidden_layers"]
        self.H = c["hidden_size"]
        self.D = c.get("head_dim") or self.H // c["num_attention_heads"]
        self.qh = c["num_attention_heads"]
        self.kvh = c["num_key_value_heads"]
        self.V = c["vocab_size"]
        self._keep = []

        def arr(name):
            a = _f32(weights[name])
            self._keep.append(a)
            return a

        def plist(suffix):
            ptrs = (_f32p * self.L)(*[_p(arr(f"model.layers.{i}.{suffix}")) for i in range(self.L)])
            self._keep.append(ptrs)
            return ptrs

        self.inv_freq = rope_inv_freq(self.D, c["rope_theta"], c.get("rope_scaling"))
        m = OrcLlama()
        m.layers, m.hidden, m.inter = self.L, self.H, c["intermediate_size"]
        m.qh, m.kvh, m.head_dim, m.vocab = self.qh, self.kvh, self.D, self.V
        m.eps = c["rms_norm_eps"]
        m.embed = _p(arr("model.embed_tokens.weight"))
        m.final_norm = _p(arr("model.norm.weight"))
        m.input_norm = plist("input_layernorm.weight")
        m.q_proj = plist("self_attn.q_proj.weight")
        m.k_proj = plist("self_attn.k_proj.weight")
        m.v_proj = plist("self_attn.v_proj.weight")
        m.o_proj = plist("self_attn.o_proj.weight")
        m.post_norm = plist("post_attention_layernorm.weight")
        m.gate_proj = plist("mlp.gate_proj.weight")
        m.up_proj = plist("mlp.up_proj.weight")
        m.down_proj = plist("mlp.down_proj.weight")
        m.inv_freq = _p(self.inv_freq)
        self.m = m

    def new_cache(self, cap):
        shape = (self.L, self.kvh, cap, self.D)
        return np.zeros(shape, np.float32), np.zeros(shape, np.float32)

    def forward(self, ids, pos, kc, vc, trace=False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        n = ids.size
        logits = np.empty(self.V, np.float32)
        tr = np.empty((self.L + 1, n, self.H), np.float32) if trace else None
        lib().orc_llama_forward(ctypes.byref(self.m), _p(ids, _i32p), n, pos, _p(kc), _p(vc), kc.shape[2],
                                _p(tr) if trace else None, _p(logits))
        return (logits, tr) if trace else logits

    def greedy(self, prompt, steps, cap=None):
        cap = cap or (len(prompt) + steps + 1)
        kc, vc = self.new_cache(cap)
        logits = self.forward(prompt, 0, kc, vc)
        out = [argmax(logits)]
        pos = len(prompt)
        while len(out) < steps:
            logits = self.forward([out[-1]], pos, kc, vc)
            pos += 1
            out.append(argmax(logits))
        return out

    def decode_batch(self, ids, pos, kc, vc):
        """One batched decode step; kc/vc [B, L, kvh, cap, D]."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pos = np.ascontiguousarray(pos, dtype=np.int32)
        B = ids.size
        logits = np.empty((B, self.V), np.float32)
        lib().orc_llama_decode_batch(ctypes.byref(self.m), _p(ids, _i32p), _p(pos, _i32p), B, _p(kc), _p(vc),
                                     kc.shape[3], _p(logits))
        return logits
