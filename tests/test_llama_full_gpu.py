"""Full-size random-init Llama-3.2-1B (OPWPACK1 float32 pack, N(0, 0.02)
weights, seed 1234, generated once per box) — benchmark config C2 parity:

* the accurate (fp32) session path gives the same first 32 greedy tokens
  after a 128-token random prompt as the CPU oracle and as the reference's own
  CUDA library (oracle/_ref/libopworks_llama_ref.so, built from the reference
  sources) on the same pack;
* the fast (bf16) path's logits stay within the GEMM tolerance of the
  fp32 path (max-abs <= 2e-2 on the logits);
* a bs32 decode step of the batch engine equals 32 single-sequence steps.
"""

import ctypes
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LLAMA = os.path.join(ROOT, "oracle", "_ref", "libopworks_llama_ref.so")
STEPS = 32


@pytest.fixture(scope="module")
def pack_path():
    from opworks_b200 import pack

    return pack.ensure_random_llama_pack()


@pytest.fixture(scope="module")
def prompt():
    return np.random.default_rng(5).integers(0, 128256, 128).astype(np.int32).tolist()


def run_c_abi(lib, pack_path, prompt, steps, logits_out=None):
    """prefill + greedy decode through an OpWorks-style C ABI library."""
    lib.opw_llama_load.restype = ctypes.c_void_p
    lib.opw_llama_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_create_session.restype = ctypes.c_void_p
    lib.opw_llama_create_session.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_prefill.restype = ctypes.c_int32
    lib.opw_llama_prefill.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                      ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_decode_step.restype = ctypes.c_int32
    lib.opw_llama_decode_step.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_last_logits.restype = ctypes.c_int
    lib.opw_llama_last_logits.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                                          ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_destroy_session.argtypes = [ctypes.c_void_p]
    lib.opw_llama_free.argtypes = [ctypes.c_void_p]
    err = ctypes.create_string_buffer(512)
    m = lib.opw_llama_load(pack_path.encode(), err, 512)
    assert m, err.value
    s = lib.opw_llama_create_session(m, 2048, err, 512)
    assert s, err.value
    arr = (ctypes.c_int32 * len(prompt))(*prompt)
    tok = lib.opw_llama_prefill(s, arr, len(prompt), err, 512)
    assert tok >= 0, err.value
    if logits_out is not None:
        lib.opw_llama_last_logits(s, logits_out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), logits_out.size,
                                  err, 512)
    out = [tok]
    while len(out) < steps:
        tok = lib.opw_llama_decode_step(s, tok, err, 512)
        assert tok >= 0, err.value
        out.append(tok)
    lib.opw_llama_destroy_session(s)
    lib.opw_llama_free(m)
    return out


@pytest.fixture(scope="module")
def ours(pack_path, prompt):
    from opworks_b200 import llama

    logits = np.empty(128256, np.float32)
    toks = run_c_abi(llama.lib(), pack_path, prompt, STEPS, logits)
    return toks, logits


def test_greedy_parity_vs_oracle(pack_path, prompt, ours):
    from opworks_b200 import pack

    manifest, tensors = pack.read_pack(pack_path)
    m = oracle.Llama(manifest["config"], tensors)
    kc, vc = m.new_cache(len(prompt) + STEPS + 1)
    logits = m.forward(prompt, 0, kc, vc)
    got_tokens, got_logits = ours
    err = np.max(np.abs(got_logits - logits))
    assert err <= 1e-3, err  # fp32 path: hidden states agree to ~1e-6 relative
    want = [oracle.argmax(logits)]
    pos = len(prompt)
    while len(want) < STEPS:
        logits = m.forward([want[-1]], pos, kc, vc)
        pos += 1
        want.append(oracle.argmax(logits))
    assert got_tokens == want


def test_greedy_parity_vs_reference_cuda(pack_path, prompt, ours):
    if not os.path.exists(REF_LLAMA):
        pytest.skip("reference library was not built (oracle/_ref)")
    ref = ctypes.CDLL(REF_LLAMA)
    want = run_c_abi(ref, pack_path, prompt, STEPS)
    assert ours[0] == want


def test_fast_path_logits_within_gemm_tolerance(pack_path, prompt, ours):
    from opworks_b200.llama import LlamaBatch, Model

    with Model(pack_path, weight_sets=1) as m, LlamaBatch(m, 1, 256, "fast") as b:
        b.prefill(0, prompt)
        fast = b.logits(0)
    err = np.max(np.abs(fast - ours[1]))
    assert err <= 2e-2, err


def test_batched_decode_equals_single(pack_path):
    from opworks_b200.llama import LlamaBatch, Model

    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, 128256, int(n)).tolist() for n in rng.integers(16, 200, 32)]
    with Model(pack_path, weight_sets=1) as m:
        with LlamaBatch(m, 32, 256, "fast", prefill_rows=256) as b:
            first = [b.prefill(i, p) for i, p in enumerate(prompts)]
            out = b.decode(list(range(32)), first)
            batch_logits = b.logits(5)
        with LlamaBatch(m, 1, 256, "fast", prefill_rows=256) as one:
            for i in (0, 5, 31):
                one.reset(0)
                t = one.prefill(0, prompts[i])
                assert t == first[i]
                nxt = one.decode([0], [t])[0]
                assert nxt == out[i]
                if i == 5:
                    err = np.max(np.abs(one.logits(0) - batch_logits))
                    assert err <= 2e-2, err


def test_fast_path_long_prompt_logits_within_gemm_tolerance(pack_path):
    """A 1024-token prompt: the fast path's prefill runs the two-SM GEMMs
    (16-bit weights x one fp16 activation term, from 256 token rows on) and tensor-core TF32
    attention; its last-row logits stay within the GEMM tolerance of
    the accurate path (fp32 weights, split-TF32 GEMMs, fp32 attention)."""
    from opworks_b200.llama import LlamaBatch, Model

    prompt = np.random.default_rng(77).integers(0, 128256, 1024).astype(np.int32).tolist()
    with Model(pack_path, weight_sets=7) as m:  # bf16 + fp32 + split-TF32 weights
        with LlamaBatch(m, 1, 1100, "accurate", prefill_rows=1024) as acc:
            t_acc = acc.prefill(0, prompt)
            ref = acc.logits(0)
        with LlamaBatch(m, 1, 1100, "fast", prefill_rows=1024) as fast:
            t_fast = fast.prefill(0, prompt)
            got = fast.logits(0)
    err = np.max(np.abs(got - ref))
    assert err <= 2e-2, err
    assert t_fast == t_acc
