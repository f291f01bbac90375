"""Python side of libopworks_llama.so (include/opworks_llama.h).

* ``LlamaGenerator`` keeps the interface of OpWorks
  examples/llama/generate.py:64-149 (``generate_ids(prompt_ids, max_new_tokens,
  temperature, top_p, seed)`` with the same capacity and EOS rules). Token
  selection runs on the GPU (fused greedy / top-p kernel); for a seed, the
  uniform of each draw comes from ``numpy.random.default_rng(seed).random()``,
  the same stream the reference's host sampler consumes, so identical logits
  give identical tokens.
* ``LlamaBatch`` drives the batched engine: many sequences per forward over a
  paged KV cache.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from . import load

_ERR_LEN = 512
P = ctypes.c_void_p
I = ctypes.c_int
I32 = ctypes.c_int32
I32P = ctypes.POINTER(ctypes.c_int32)
F = ctypes.c_float
FP = ctypes.POINTER(ctypes.c_float)
D = ctypes.c_double
DP = ctypes.POINTER(ctypes.c_double)
U64 = ctypes.c_uint64
U64P = ctypes.POINTER(ctypes.c_uint64)
S = ctypes.c_char_p

PRECISION = {"accurate": 0, "fast": 1}


def bind(lib):
    if getattr(lib, "_opw_bound", False):
        return lib
    sig = {
        "opw_llama_load": (P, [S, S, I]),
        "opw_llama_load_ex": (P, [S, ctypes.c_uint, I, S, I]),
        "opw_llama_free": (None, [P]),
        "opw_llama_create_session": (P, [P, I, S, I]),
        "opw_llama_destroy_session": (None, [P]),
        "opw_llama_reset_session": (I, [P, S, I]),
        "opw_llama_prefill": (I32, [P, I32P, I, S, I]),
        "opw_llama_decode_step": (I32, [P, I32, S, I]),
        "opw_llama_is_eos": (I, [P, I32, S, I]),
        "opw_llama_last_logits": (I, [P, FP, I, S, I]),
        "opw_llama_vocab_size": (I, [P]),
        "opw_llama_last_error": (S, []),
        "opw_llama_set_device": (I, [I]),
        "opw_llama_model_info": (I, [P, I32P, S, I]),
        "opw_llama_create_batch": (P, [P, I, I, I, I, S, I]),
        "opw_llama_create_batch_tp": (P, [P, I, I, I, I, I, ctypes.c_char_p, S, I]),
        "opw_llama_nccl_unique_id": (I, [ctypes.c_char_p, S, I]),
        "opw_llama_batch_tp_ipc_handle": (I, [P, ctypes.c_char_p, S, I]),
        "opw_llama_batch_tp_open_peers": (I, [P, ctypes.c_char_p, S, I]),
        "opw_llama_destroy_batch": (None, [P]),
        "opw_llama_batch_reset": (I, [P, I, S, I]),
        "opw_llama_batch_length": (I, [P, I]),
        "opw_llama_batch_prefill": (I, [P, I, I32P, I, F, F, D, U64, S, I]),
        "opw_llama_batch_decode": (I, [P, I, I32P, I32P, FP, FP, DP, U64P, I32P, I32P, S, I]),
        "opw_llama_batch_decode_multi": (I, [P, I, I32P, I32P, FP, FP, DP, U64P, I32P, I, I, I32P, I32P, S, I]),
        "opw_llama_batch_logits": (I, [P, I, FP, I, S, I]),
        "opw_llama_batch_kv_blocks": (I, [P, I, I32P, I, S, I]),
        "opw_llama_batch_kv_read": (I, [P, I, I, I, I, FP, FP, S, I]),
        "opw_llama_batch_kv_pool": (I, [P, I, I, I, FP, FP, S, I]),
        "opw_llama_batch_stream": (P, [P]),
        "opw_llama_batch_io_bytes": (I, [P, I, ctypes.POINTER(ctypes.c_int64)]),
        "opw_llama_batch_profile": (I, [P, I, I, FP, I32P, S, I, S, I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    lib._opw_bound = True
    return lib


def lib():
    return bind(load("libopworks_llama.so"))


def _i32(a):
    a = np.ascontiguousarray(a, dtype=np.int32)
    return a, a.ctypes.data_as(I32P)


class Model:
    """A loaded weight pack (float32 or bfloat16 OPWPACK1)."""

    def __init__(self, pack_path, weight_sets=0, max_positions=8192, device=None):
        self.lib = lib()
        self.err = ctypes.create_string_buffer(_ERR_LEN)
        if device is not None and self.lib.opw_llama_set_device(int(device)) != 0:
            raise RuntimeError(f"cannot select device {device}")
        if weight_sets or max_positions != 8192:
            self.handle = self.lib.opw_llama_load_ex(pack_path.encode(), weight_sets, max_positions, self.err,
                                                     _ERR_LEN)
        else:
            self.handle = self.lib.opw_llama_load(pack_path.encode(), self.err, _ERR_LEN)
        if not self.handle:
            raise RuntimeError(f"model load failed: {self.err.value.decode(errors='replace')}")
        info = np.zeros(8, np.int32)
        self.lib.opw_llama_model_info(self.handle, info.ctypes.data_as(I32P), self.err, _ERR_LEN)
        (self.layers, self.hidden, self.intermediate, self.q_heads, self.kv_heads, self.head_dim, self.vocab,
         self.device) = (int(v) for v in info)

    def close(self):
        if self.handle:
            self.lib.opw_llama_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def nccl_unique_id():
    """A 128-byte NCCL communicator id for LlamaBatch(tp=(rank, world, id))."""
    import opworks_b200

    lib = opworks_b200.llama_lib()
    out = ctypes.create_string_buffer(128)
    err = ctypes.create_string_buffer(_ERR_LEN)
    if lib.opw_llama_nccl_unique_id(out, err, _ERR_LEN) < 0:
        raise RuntimeError(f"nccl id failed: {err.value.decode(errors='replace')}")
    return out.raw


class LlamaBatch:
    """Batched engine: slots 0..max_batch-1 share a paged KV cache."""

    def __init__(self, model: Model, max_batch, max_seq_len, precision="fast", prefill_rows=0, tp=None):
        """tp = (rank, world, nccl_id): this process's rank of a tensor-parallel
        group (fast path; nccl_id from nccl_unique_id() on one rank)."""
        self.model = model
        self.lib = model.lib
        self.err = ctypes.create_string_buffer(_ERR_LEN)
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.tp_world = 1 if tp is None else int(tp[1])
        if tp is not None:
            rank, world, nccl_id = tp
            assert precision == "fast" and len(nccl_id) == 128
            self.handle = self.lib.opw_llama_create_batch_tp(model.handle, max_batch, max_seq_len, prefill_rows, rank,
                                                             world, bytes(nccl_id), self.err, _ERR_LEN)
        else:
            self.handle = self.lib.opw_llama_create_batch(model.handle, max_batch, max_seq_len, PRECISION[precision],
                                                          prefill_rows, self.err, _ERR_LEN)
        if not self.handle:
            raise RuntimeError(f"batch creation failed: {self.err.value.decode(errors='replace')}")
        self._out = np.zeros(max_batch, np.int32)

    def _check(self, rc, what):
        if rc < 0:
            raise RuntimeError(f"{what} failed: {self.err.value.decode(errors='replace')}")
        return rc

    def tp_ipc_handle(self):
        """128 bytes: CUDA IPC handles of this rank's receive buffer and
        counters (tensor-parallel batches), to be shared with the other ranks."""
        out = ctypes.create_string_buffer(128)
        self._check(self.lib.opw_llama_batch_tp_ipc_handle(self.handle, out, self.err, _ERR_LEN), "tp ipc handle")
        return out.raw

    def tp_open_peers(self, handles):
        """handles: every rank's tp_ipc_handle() in rank order. Switches the
        o / down reductions from NCCL to peer stores from the GEMM epilogue."""
        blob = b"".join(bytes(h) for h in handles)
        assert all(len(h) == 128 for h in handles)
        self._check(self.lib.opw_llama_batch_tp_open_peers(self.handle, blob, self.err, _ERR_LEN), "tp open peers")

    def reset(self, slot):
        self._check(self.lib.opw_llama_batch_reset(self.handle, slot, self.err, _ERR_LEN), "reset")

    def length(self, slot):
        return self.lib.opw_llama_batch_length(self.handle, slot)

    def prefill(self, slot, ids, temperature=0.0, top_p=1.0, uniform=-1.0, seed=0):
        arr, ptr = _i32(ids)
        return self._check(self.lib.opw_llama_batch_prefill(self.handle, slot, ptr, arr.size, temperature, top_p,
                                                            uniform, seed, self.err, _ERR_LEN), "prefill")

    def decode(self, slots, prev, temperature=None, top_p=None, uniforms=None, seeds=None, steps=None):
        slots_a, slots_p = _i32(slots)
        prev_a, prev_p = _i32(prev)
        n = slots_a.size
        keep = []

        def opt(a, dtype, ptype):
            if a is None:
                return None
            a = np.ascontiguousarray(np.broadcast_to(a, (n,)), dtype=dtype)
            keep.append(a)
            return a.ctypes.data_as(ptype)

        out = self._out[:n]
        self._check(self.lib.opw_llama_batch_decode(
            self.handle, n, slots_p, prev_p, opt(temperature, np.float32, FP), opt(top_p, np.float32, FP),
            opt(uniforms, np.float64, DP), opt(seeds, np.uint64, U64P), opt(steps, np.int32, I32P),
            out.ctypes.data_as(I32P), self.err, _ERR_LEN), "decode")
        return out.copy()

    def decode_multi(self, slots, prev, steps, temperature=None, top_p=None, uniforms=None, seeds=None, steps0=None,
                     eos_id=-1):
        """`steps` decode steps with no host round trip per step. Returns
        (tokens [steps][n] with -1 after a row's eos, counts [n]). `uniforms`,
        when given, is [steps][n]."""
        slots_a, slots_p = _i32(slots)
        prev_a, prev_p = _i32(prev)
        n = slots_a.size
        keep = []

        def opt(a, dtype, ptype, shape):
            if a is None:
                return None
            a = np.ascontiguousarray(np.broadcast_to(a, shape), dtype=dtype)
            keep.append(a)
            return a.ctypes.data_as(ptype)

        out = np.empty((steps, n), np.int32)
        counts = np.empty(n, np.int32)
        self._check(self.lib.opw_llama_batch_decode_multi(
            self.handle, n, slots_p, prev_p, opt(temperature, np.float32, FP, (n,)), opt(top_p, np.float32, FP, (n,)),
            opt(uniforms, np.float64, DP, (steps, n)), opt(seeds, np.uint64, U64P, (n,)),
            opt(steps0, np.int32, I32P, (n,)), steps, eos_id, out.ctypes.data_as(I32P), counts.ctypes.data_as(I32P),
            self.err, _ERR_LEN), "decode_multi")
        return out, counts

    def stream(self):
        """The engine's cudaStream_t as an integer."""
        return self.lib.opw_llama_batch_stream(self.handle) or 0

    def io_bytes(self, n):
        out = np.zeros(2, np.int64)
        self.lib.opw_llama_batch_io_bytes(self.handle, n, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)))
        return int(out[0]), int(out[1])

    def profile(self, n, iters=3):
        """[(label, ms per step, launches per step)] of the last decode step of n rows."""
        k = 32
        ms = np.zeros(k, np.float32)
        launches = np.zeros(k, np.int32)
        labels = ctypes.create_string_buffer(32 * k)
        cnt = self._check(self.lib.opw_llama_batch_profile(self.handle, n, iters, ms.ctypes.data_as(FP),
                                                           launches.ctypes.data_as(I32P), labels, k, self.err,
                                                           _ERR_LEN), "profile")
        raw = labels.raw
        return [(raw[32 * i:32 * i + 32].split(b"\0")[0].decode(), float(ms[i]), int(launches[i]))
                for i in range(cnt)]

    def logits(self, row):
        out = np.empty(self.model.vocab, np.float32)
        self._check(self.lib.opw_llama_batch_logits(self.handle, row, out.ctypes.data_as(FP), out.size, self.err,
                                                    _ERR_LEN), "logits")
        return out

    def kv_blocks(self, slot):
        """Physical KV block ids of `slot` (the device copy of its block table)."""
        cap = (self.max_seq_len + 15) // 16
        out = np.zeros(cap, np.int32)
        n = self._check(self.lib.opw_llama_batch_kv_blocks(self.handle, slot, out.ctypes.data_as(I32P), cap, self.err,
                                                           _ERR_LEN), "kv blocks")
        return out[:n].copy()

    def kv_read(self, slot, layer, pos0, n):
        """(K, V) of positions [pos0, pos0 + n) of `slot` in `layer`, read
        through the block table: two [n][kv_heads][head_dim] float32 arrays."""
        shape = (n, self.model.kv_heads // self.tp_world, self.model.head_dim)
        k = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        self._check(self.lib.opw_llama_batch_kv_read(self.handle, slot, layer, pos0, n, k.ctypes.data_as(FP),
                                                     v.ctypes.data_as(FP), self.err, _ERR_LEN), "kv read")
        return k, v

    def kv_pool(self, layer, block0=0, nblocks=None):
        """Raw physical blocks of `layer`: (K, V) as [blocks][kv_heads][16][head_dim]."""
        total = self._check(self.lib.opw_llama_batch_kv_pool(self.handle, layer, 0, 0, None, None, self.err, _ERR_LEN),
                            "kv pool")
        if nblocks is None:
            nblocks = total - block0
        shape = (nblocks, self.model.kv_heads // self.tp_world, 16, self.model.head_dim)
        k = np.empty(shape, np.float32)
        v = np.empty(shape, np.float32)
        self._check(self.lib.opw_llama_batch_kv_pool(self.handle, layer, block0, nblocks, k.ctypes.data_as(FP),
                                                     v.ctypes.data_as(FP), self.err, _ERR_LEN), "kv pool")
        return k, v

    def close(self):
        if self.handle:
            self.lib.opw_llama_destroy_batch(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class LlamaGenerator:
    """Drop-in for OpWorks' LlamaGenerator (examples/llama/generate.py:64-149)
    with sampling on the device."""

    def __init__(self, pack_path, lib_path=None, max_seq_len=2048, precision=None):
        del lib_path  # the in-tree library is always used
        self.model = Model(pack_path)
        with open(pack_path, "rb") as f:
            head = f.read(4096)
        is_bf16 = b'"dtype": "bfloat16"' in head
        self.precision = precision or ("fast" if is_bf16 else "accurate")
        self.batch = LlamaBatch(self.model, 1, max_seq_len, self.precision)
        self.max_seq_len = max_seq_len
        self._vocab = self.model.vocab
        eos = np.array([128001, 128008, 128009])
        self._eos = set(int(x) for x in eos)
        self._eos_from_model = None

    def _is_eos(self, tok):
        # the session ABI exposes the manifest's EOS ids; keep one session for it
        if self._eos_from_model is None:
            err = ctypes.create_string_buffer(_ERR_LEN)
            sess = self.model.lib.opw_llama_create_session(self.model.handle, 1, err, _ERR_LEN)
            if not sess:
                raise RuntimeError(err.value.decode(errors="replace"))
            self._eos_session = sess
            self._eos_from_model = True
        rc = self.model.lib.opw_llama_is_eos(self._eos_session, int(tok), None, 0)
        if rc < 0:
            raise RuntimeError("is_eos failed")
        return rc == 1

    def generate_ids(self, prompt_ids, max_new_tokens, temperature=0.0, top_p=1.0, seed=None):
        if len(prompt_ids) + max_new_tokens > self.max_seq_len:
            raise ValueError(f"prompt ({len(prompt_ids)}) + max_new_tokens ({max_new_tokens}) "
                             f"exceeds capacity {self.max_seq_len}")
        sample = temperature > 0.0
        rng = np.random.default_rng(seed) if sample else None
        self.batch.reset(0)
        t = float(temperature) if sample else 0.0
        u = rng.random() if sample else -1.0
        tok = self.batch.prefill(0, list(prompt_ids), t, float(top_p), u)
        out = []
        for _ in range(max_new_tokens):
            out.append(int(tok))
            if self._is_eos(tok):
                break
            if len(prompt_ids) + len(out) >= self.max_seq_len and len(out) < max_new_tokens:
                break
            if len(out) == max_new_tokens:
                break
            u = rng.random() if sample else -1.0
            tok = int(self.batch.decode([0], [tok], temperature=t, top_p=float(top_p), uniforms=u)[0])
        return out

    def close(self):
        if getattr(self, "_eos_session", None):
            self.model.lib.opw_llama_destroy_session(self._eos_session)
            self._eos_session = None
        self.batch.close()
        self.model.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
