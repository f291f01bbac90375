"""A bfloat16 OPWPACK1 pack (the reference's LlamaModelBF16 path,
src/llama_c_api.cu:59-63 and tests/model/llama_bf16_test.cu) through the
reference's 11-symbol session ABI: the same random-init Llama-3.2-1B draw,
each weight rounded to bf16.

* prefill logits within the GEMM tolerance (2e-2 max-abs) of the CPU oracle
  computing in double on the pack's exact bf16 values;
* greedy generation against two teachers, the oracle and the reference's own
  CUDA library on the same pack, with the reference's bf16 rule
  (tests/model/model_test_body.cuh:21,246-264): a divergence from the teacher
  is allowed only where our top-1 / top-2 logit margin, on the teacher's
  prefix, is at most 0.05.
"""

import ctypes
import os

import numpy as np
import pytest

import oracle
from test_llama_full_gpu import REF_LLAMA, run_c_abi

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

STEPS = 32
MARGIN = 0.05  # kBf16MarginLimit of the reference's model tests


@pytest.fixture(scope="module")
def bf16_pack():
    from opworks_b200 import pack

    return pack.ensure_random_llama_pack(dtype="bfloat16")


@pytest.fixture(scope="module")
def prompt():
    return np.random.default_rng(5).integers(0, 128256, 128).astype(np.int32).tolist()


@pytest.fixture(scope="module")
def ours(bf16_pack, prompt):
    from opworks_b200 import llama

    logits = np.empty(128256, np.float32)
    return run_c_abi(llama.lib(), bf16_pack, prompt, STEPS, logits), logits


def _margin_on_prefix(pack_path, prompt, prefix):
    """Our top-1 minus top-2 logit after prefilling prompt + prefix (teacher forcing)."""
    from opworks_b200 import llama

    logits = np.empty(128256, np.float32)
    run_c_abi(llama.lib(), pack_path, list(prompt) + list(prefix), 1, logits)
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0])


def _check_against_teacher(pack_path, prompt, got, want):
    step = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    if step is None:
        return None
    margin = _margin_on_prefix(pack_path, prompt, want[:step])
    assert margin <= MARGIN, f"diverged at step {step} with margin {margin:.4f}"
    return step, margin


def test_bf16_pack_logits_and_greedy_vs_oracle(bf16_pack, prompt, ours):
    from opworks_b200 import pack

    manifest, tensors = pack.read_pack(bf16_pack)
    weights = {k: (np.asarray(v).astype(np.uint32) << 16).view(np.float32) for k, v in tensors.items()}
    m = oracle.Llama(manifest["config"], weights)
    kc, vc = m.new_cache(len(prompt) + STEPS + 1)
    logits = m.forward(prompt, 0, kc, vc)
    got_tokens, got_logits = ours
    err = float(np.max(np.abs(got_logits - logits)))
    want = [oracle.argmax(logits)]
    pos = len(prompt)
    while len(want) < STEPS:
        want.append(oracle.argmax(m.forward([want[-1]], pos, kc, vc)))
        pos += 1
    div = _check_against_teacher(bf16_pack, prompt, got_tokens, want)
    print(f"PARITY bf16_pack logits_max_abs_vs_oracle={err:.3e} divergence_vs_oracle={div}")
    assert err <= 2e-2, err


def test_bf16_pack_greedy_vs_reference_cuda(bf16_pack, prompt, ours):
    if not os.path.exists(REF_LLAMA):
        pytest.skip("reference library was not built (oracle/_ref)")
    want = run_c_abi(ctypes.CDLL(REF_LLAMA), bf16_pack, prompt, STEPS)
    div = _check_against_teacher(bf16_pack, prompt, ours[0], want)
    print(f"PARITY bf16_pack divergence_vs_reference_library={div}")
