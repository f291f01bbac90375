"""Llama runtime through libopworks_llama.so (include/opworks_llama.h) on a
small Llama (2 layers, hidden 512, 8 q heads / 2 kv heads, head_dim 64,
vocab 2048, llama3 RoPE) whose weights come from tests/golden/inputs.py.

Checks follow the reference's model tests (tests/model/model_test_body.cuh):
logits against transformers (fp32 thresholds nrmse <= 1e-3, cos >= 0.9999),
greedy continuation equal to transformers' generate, KV consistency
decode(L) vs prefill(L+1) with nrmse <= 1e-5, reset isolation, concurrent
sessions, the C-ABI edge cases of test_edges.py, plus the batch engine
(paged KV, CUDA-graph decode, device sampler) against the oracle."""

import ctypes
import os

import numpy as np
import pytest

import inputs
import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ERR = 256


def stats(a, e):
    a, e = np.asarray(a, np.float64).ravel(), np.asarray(e, np.float64).ravel()
    nrmse = np.sqrt(np.mean((a - e) ** 2)) / max(np.sqrt(np.mean(e**2)), 1e-6)
    cos = a @ e / max(np.linalg.norm(a) * np.linalg.norm(e), 1e-30)
    return nrmse, cos


@pytest.fixture(scope="module")
def tiny_pack(tmp_path_factory):
    from opworks_b200 import pack

    path = str(tmp_path_factory.mktemp("packs") / "tiny.pack")
    w = inputs.tiny_weights()
    specs = [(n, s) for n, s, _ in pack.llama_tensor_specs(inputs.TINY_CFG)]
    pack.write_pack(path, specs, lambda n, s: w[n], extra={"config": inputs.TINY_CFG, "eos_token_ids": [2046]},
                    aliases={"lm_head.weight": "model.embed_tokens.weight"})
    return path


@pytest.fixture(scope="module")
def lib():
    from opworks_b200 import llama

    return llama.lib()


@pytest.fixture(scope="module")
def model(lib, tiny_pack):
    err = ctypes.create_string_buffer(ERR)
    m = lib.opw_llama_load(tiny_pack.encode(), err, ERR)
    assert m, err.value
    yield m
    lib.opw_llama_free(m)


@pytest.fixture(scope="module")
def orc():
    return oracle.Llama(inputs.TINY_CFG, inputs.tiny_weights())


class Session:
    def __init__(self, lib, model, cap=2048):
        self.lib = lib
        self.err = ctypes.create_string_buffer(ERR)
        self.h = lib.opw_llama_create_session(model, cap, self.err, ERR)
        assert self.h, self.err.value

    def prefill(self, ids):
        a = (ctypes.c_int32 * max(1, len(ids)))(*ids)
        return self.lib.opw_llama_prefill(self.h, a, len(ids), self.err, ERR)

    def decode(self, tok):
        return self.lib.opw_llama_decode_step(self.h, tok, self.err, ERR)

    def logits(self):
        v = self.lib.opw_llama_vocab_size(self.h)
        out = np.empty(v, np.float32)
        rc = self.lib.opw_llama_last_logits(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), v,
                                            self.err, ERR)
        assert rc == 0, self.err.value
        return out

    def reset(self):
        assert self.lib.opw_llama_reset_session(self.h, self.err, ERR) == 0

    def close(self):
        self.lib.opw_llama_destroy_session(self.h)


def greedy(sess, prompt, steps):
    tok = sess.prefill(prompt)
    out = []
    for i in range(steps):
        out.append(tok)
        if i + 1 < steps:
            tok = sess.decode(tok)
    return out


def test_session_matches_transformers(lib, model):
    g = np.load(os.path.join(GOLD, "tiny_llama.npz"))
    s = Session(lib, model)
    tok = s.prefill(inputs.TINY_PROMPT)
    nrmse, cos = stats(s.logits(), g["logits"])
    assert nrmse <= 1e-3 and cos >= 0.9999, (nrmse, cos)
    assert tok == int(g["greedy"][0])
    s.reset()
    assert greedy(s, inputs.TINY_PROMPT, inputs.TINY_STEPS) == g["greedy"].tolist()
    s.close()


def test_kv_consistency_sweep(lib, model, orc):
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 2048, 140).tolist()
    for L in (1, 2, 31, 32, 33, 127, 128, 129):
        a = Session(lib, model)
        a.prefill(ids[:L])
        a.decode(ids[L])
        la = a.logits()
        b = Session(lib, model)
        b.prefill(ids[:L + 1])
        lb = b.logits()
        nrmse, cos = stats(la, lb)
        assert nrmse <= 1e-5 and cos >= 0.999999, (L, nrmse, cos)
        if L in (33, 129):
            kc, vc = orc.new_cache(L + 2)
            want = orc.forward(ids[:L + 1], 0, kc, vc)
            nrmse, cos = stats(lb, want)
            assert nrmse <= 1e-4 and cos >= 0.99999, (L, nrmse, cos)
        a.close()
        b.close()


def test_reset_isolation_and_concurrent_sessions(lib, model):
    p = inputs.TINY_PROMPT
    s = Session(lib, model)
    first = greedy(s, p, 6)
    s.reset()
    assert greedy(s, p, 6) == first
    s.close()
    s1, s2 = Session(lib, model), Session(lib, model)
    t1, t2 = s1.prefill(p[:6]), s2.prefill(p[6:])
    for _ in range(8):
        t1, t2 = s1.decode(t1), s2.decode(t2)
    r1, r2 = Session(lib, model), Session(lib, model)
    u1 = r1.prefill(p[:6])
    for _ in range(8):
        u1 = r1.decode(u1)
    u2 = r2.prefill(p[6:])
    for _ in range(8):
        u2 = r2.decode(u2)
    assert (t1, t2) == (u1, u2)
    for x in (s1, s2, r1, r2):
        x.close()


def test_c_abi_edges(lib, model):
    # tests/model/test_edges.py: OOB id, over capacity, empty prompt, reuse after errors
    s = Session(lib, model, cap=16)
    assert s.prefill([]) == -1 and b"at least one token" in s.err.value
    assert s.prefill([2048]) == -1 and b"vocabulary" in s.err.value
    assert lib.opw_llama_last_error() == s.err.value
    assert s.prefill(list(range(17))) == -1 and b"capacity" in s.err.value
    tok = s.prefill(list(range(15)))
    assert tok >= 0
    assert s.prefill([1]) == -1 and b"fresh session" in s.err.value
    assert s.decode(-1) == -1
    assert s.decode(tok) >= 0  # 16th position: exactly at capacity
    assert s.decode(tok) == -1 and b"capacity" in s.err.value
    bad = np.empty(10, np.float32)
    assert lib.opw_llama_last_logits(s.h, bad.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 10, s.err, ERR) == -1
    assert lib.opw_llama_is_eos(s.h, 2046, s.err, ERR) == 1
    assert lib.opw_llama_is_eos(s.h, 5, s.err, ERR) == 0
    s.reset()
    assert s.prefill([1, 2, 3]) >= 0  # usable after errors
    s.close()
    err = ctypes.create_string_buffer(ERR)
    assert not lib.opw_llama_create_session(model, 0, err, ERR)
    assert not lib.opw_llama_load(b"/nonexistent.pack", err, ERR)


def test_batch_engine_fast_and_accurate(tiny_pack, orc):
    from opworks_b200.llama import LlamaBatch, Model

    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 2048, n).tolist() for n in (12, 40, 77)]
    with Model(tiny_pack) as m:
        for prec in ("accurate", "fast"):
            with LlamaBatch(m, 4, 256, prec) as b:
                toks = [b.prefill(i, p) for i, p in enumerate(prompts)]
                for i, p in enumerate(prompts):
                    b.reset(i)
                    toks[i] = b.prefill(i, p)
                    kc, vc = orc.new_cache(len(p) + 1)
                    want = orc.forward(p, 0, kc, vc)
                    nrmse, cos = stats(b.logits(0), want)
                    if prec == "accurate":
                        assert nrmse <= 1e-4 and cos >= 0.99999, (prec, nrmse)
                    else:
                        assert nrmse <= 1e-2 and cos >= 0.999, (prec, nrmse)
                # batched decode == one slot at a time (graph path, 3 rows)
                seq = [[t] for t in toks]
                for _ in range(6):
                    nxt = b.decode([0, 1, 2], [s[-1] for s in seq])
                    for i in range(3):
                        seq[i].append(int(nxt[i]))
                with LlamaBatch(m, 1, 256, prec) as one:
                    for i, p in enumerate(prompts):
                        one.reset(0)
                        t = one.prefill(0, p)
                        got = [t]
                        for _ in range(6):
                            t = int(one.decode([0], [t])[0])
                            got.append(t)
                        assert got == seq[i], (prec, i)


def test_chunked_prefill_equals_whole(tiny_pack):
    from opworks_b200.llama import LlamaBatch, Model

    ids = np.random.default_rng(9).integers(0, 2048, 50).tolist()
    with Model(tiny_pack) as m:
        with LlamaBatch(m, 1, 128, "accurate") as whole, LlamaBatch(m, 1, 128, "accurate", prefill_rows=7) as ch:
            a = whole.prefill(0, ids)
            b = ch.prefill(0, ids)
            nrmse, _ = stats(whole.logits(0), ch.logits(0))
            assert a == b and nrmse <= 1e-5, nrmse


def test_engine_sampling_uses_the_reference_rule(tiny_pack):
    from opworks_b200.llama import LlamaBatch, Model

    ids = inputs.TINY_PROMPT
    with Model(tiny_pack) as m, LlamaBatch(m, 2, 64, "accurate") as b:
        for u in (0.0, 0.13, 0.5, 0.77, 0.999):
            b.reset(0)
            tok = b.prefill(0, ids, temperature=0.7, top_p=0.9, uniform=u)
            assert tok == oracle.top_p_sample(b.logits(0), 0.7, 0.9, u)
        # decode rows sample with their own uniforms
        b.reset(0)
        b.reset(1)
        t0 = b.prefill(0, ids[:5])
        t1 = b.prefill(1, ids[5:])
        us = [0.31, 0.62]
        out = b.decode([0, 1], [t0, t1], temperature=[0.7, 1.3], top_p=[0.9, 0.5], uniforms=us)
        assert out[0] == oracle.top_p_sample(b.logits(0), 0.7, 0.9, us[0])
        assert out[1] == oracle.top_p_sample(b.logits(1), 1.3, 0.5, us[1])
        # counter-based draws are reproducible per (seed, step)
        b.reset(0)
        t = b.prefill(0, ids, temperature=0.8, top_p=0.95, seed=7)
        b.reset(1)
        t2 = b.prefill(1, ids, temperature=0.8, top_p=0.95, seed=7)
        assert t == t2


def test_generator_drop_in(tiny_pack):
    from opworks_b200.llama import LlamaGenerator

    g = np.load(os.path.join(GOLD, "tiny_llama.npz"))
    with LlamaGenerator(tiny_pack, max_seq_len=64) as gen:
        assert gen.generate_ids(inputs.TINY_PROMPT, inputs.TINY_STEPS) == g["greedy"].tolist()
        assert gen.generate_ids(inputs.TINY_PROMPT, 0) == []
        assert len(gen.generate_ids(inputs.TINY_PROMPT, 1)) == 1
        a = gen.generate_ids(inputs.TINY_PROMPT, 10, temperature=0.7, top_p=0.9, seed=3)
        b = gen.generate_ids(inputs.TINY_PROMPT, 10, temperature=0.7, top_p=0.9, seed=3)
        assert a == b and len(a) >= 1
        with pytest.raises(ValueError):
            gen.generate_ids(inputs.TINY_PROMPT, 60)
