"""Pins the CPU oracle (oracle/oracle.cpp) before anything is compared with it:
against the closed-form expectations of the reference's tests/unit/framework.cu
and against golden vectors produced by the reference's own Python math,
transformers' Llama forward and the reference host sampler
(tests/golden/make_golden.py)."""

import math
import os

import numpy as np
import pytest

import inputs
import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def close(a, e, tol=1e-5):
    a, e = np.asarray(a, np.float64), np.asarray(e, np.float64)
    assert np.all(np.isfinite(a))
    assert np.all(np.abs(a - e) <= tol * (1 + np.abs(e))), float(np.max(np.abs(a - e) / (1 + np.abs(e))))


def test_framework_closed_forms():
    # tests/unit/framework.cu:182-223
    x = np.array([[-2, -1, 0, 1, 2], [3, 4, 5, 6, 7]], np.float32)
    den = sum(math.exp(j - 4) for j in range(5))
    close(oracle.softmax(x), [[math.exp(i - 4) / den for i in range(5)]] * 2)
    ln = oracle.layer_norm(x, np.full(5, 2, np.float32), np.full(5, 1, np.float32), 1e-5)
    close(ln, [[(i - 2) * 2 / math.sqrt(2 + 1e-5) + 1 for i in range(5)]] * 2)
    a = np.array([i % 7 - 3 for i in range(15)], np.float32).reshape(3, 5)
    b = np.array([i % 5 - 2 for i in range(35)], np.float32).reshape(5, 7)
    close(oracle.mat_mul(a, b, epilogue=2, param=2.0), 2 * (a.astype(np.float64) @ b))
    close(oracle.mat_mul(np.zeros((3, 0), np.float32), np.zeros((0, 7), np.float32)), np.zeros((3, 7)))
    for n in (0, 1, 31, 32, 33, 255, 256, 257, 4099):
        assert oracle.reduce_sum(np.ones(n, np.float32)) == n


def test_ops_against_reference_math():
    g = np.load(os.path.join(GOLD, "ops_golden.npz"))
    x = inputs.op_inputs()
    close(oracle.rms_norm(x["rms.x"], x["rms.w"], inputs.EPS), g["rms.out"], 1e-5)
    inv = oracle.rope_inv_freq(inputs.D, inputs.THETA, inputs.ROPE_SCALING)
    close(inv, g["rope.inv_freq"], 1e-6)
    close(oracle.rope(x["rope.q"], inv, inputs.QH, inputs.D, 29), g["rope.q_out"], 1e-5)
    close(oracle.rope(x["rope.k"], inv, inputs.KVH, inputs.D, 29), g["rope.k_out"], 1e-5)
    close(oracle.attention(x["attn.q"], x["attn.k"], x["attn.v"]), g["attn.out"], 1e-5)
    close(oracle.attention(x["attn.qd"], x["attn.k"], x["attn.v"]), g["attn.out_decode"], 1e-5)
    close(oracle.swiglu(x["swiglu.g"], x["swiglu.u"]), g["swiglu.out"], 1e-5)
    close(oracle.linear(x["lin.x"], x["lin.w"]), g["lin.out"], 1e-5)
    close(oracle.linear(x["gemv.x"], x["gemv.w"]), g["gemv.out"], 1e-5)
    assert oracle.argmax(x["argmax.x"]) == int(g["argmax.out"][0])


def test_tiny_llama_against_transformers():
    g = np.load(os.path.join(GOLD, "tiny_llama.npz"))
    m = oracle.Llama(inputs.TINY_CFG, inputs.tiny_weights())
    kc, vc = m.new_cache(64)
    logits, trace = m.forward(inputs.TINY_PROMPT, 0, kc, vc, trace=True)
    for i in range(trace.shape[0]):
        err = np.linalg.norm(trace[i] - g["hidden"][i]) / np.linalg.norm(g["hidden"][i])
        assert err < 1e-5, (i, err)
    err = np.max(np.abs(logits - g["logits"]))
    assert err < 1e-3 * max(1.0, np.max(np.abs(g["logits"]))), err
    assert m.greedy(inputs.TINY_PROMPT, inputs.TINY_STEPS) == g["greedy"].tolist()


def test_kv_decode_equals_prefill_in_oracle():
    m = oracle.Llama(inputs.TINY_CFG, inputs.tiny_weights())
    p = inputs.TINY_PROMPT
    kc, vc = m.new_cache(32)
    m.forward(p[:-1], 0, kc, vc)
    a = m.forward(p[-1:], len(p) - 1, kc, vc)
    kc2, vc2 = m.new_cache(32)
    b = m.forward(p, 0, kc2, vc2)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", inputs.SAMPLER_CASES)
def test_sampler_against_reference_host_sampler(case):
    vocab, scale, temp, top_p, seed = case
    want = np.load(os.path.join(GOLD, "sampler_golden.npz"))[f"case{seed}"]
    logits = inputs.sampler_logits(vocab, scale, seed)
    rng = np.random.default_rng(seed)
    got = [oracle.top_p_sample(logits, temp, top_p, rng.random()) for _ in range(inputs.SAMPLER_DRAWS)]
    assert got == want.tolist()
