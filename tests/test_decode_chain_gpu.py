"""The persistent decode chain (include/ops/decode_chain.cuh, OPWORKS_CHAIN=1):
one launch per layer runs the O, gate/up and down projections and the next
layer's QKV as phases of a grid of one CTA per SM. It must give what the
four GEMM kernels give (the same 16-bit operands, fp32 accumulation; only the
split-K summation order differs) at batch sizes 32, 7 and 1, and leave its
phase counters re-armed for the next launch (several steps in a row)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

STEPS = 4


@pytest.fixture(scope="module")
def pack_path():
    from opworks_b200 import pack

    return pack.ensure_random_llama_pack()


def _run(pack_path, prompts, chain, monkeypatch):
    from opworks_b200.llama import LlamaBatch, Model

    if chain:
        monkeypatch.setenv("OPWORKS_CHAIN", "1")
    else:
        monkeypatch.delenv("OPWORKS_CHAIN", raising=False)
    n = len(prompts)
    with Model(pack_path, weight_sets=1) as m:
        with LlamaBatch(m, n, 256, "fast", prefill_rows=256) as b:
            prev = [b.prefill(i, p) for i, p in enumerate(prompts)]
            tokens, logits = [list(prev)], []
            for _ in range(STEPS):
                prev = b.decode(list(range(n)), prev)
                tokens.append(list(prev))
                logits.append(np.stack([b.logits(i) for i in range(n)]))
    return tokens, logits


@pytest.mark.parametrize("batch", [32, 7, 1])
def test_decode_chain_matches_kernel_path(pack_path, batch, monkeypatch):
    rng = np.random.default_rng(40 + batch)
    prompts = [rng.integers(0, 128256, int(n)).tolist() for n in rng.integers(16, 200, batch)]
    want_tokens, want_logits = _run(pack_path, prompts, False, monkeypatch)
    got_tokens, got_logits = _run(pack_path, prompts, True, monkeypatch)
    err = max(float(np.max(np.abs(g - w))) for g, w in zip(got_logits, want_logits))
    print(f"PARITY decode_chain batch={batch} logits_max_abs_vs_kernel_path={err:.3e}")
    # the same operands and products; split-K partial sums add in another order
    assert err <= 2e-3, err
    assert got_tokens == want_tokens
