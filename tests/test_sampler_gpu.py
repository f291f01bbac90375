"""The fused top-p / argmax sampler (ops/llama_kernels.cuh sample_kernel),
called through libopworks_ops.so's opw_sample, against the pinned oracle
restatement of the reference's host sampler (examples/llama/generate.py:83-109,
numpy Generator.choice with the same uniform). Token ids are integers: the
check is bit-exact."""

import numpy as np
import pytest

import inputs
import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ops():
    import opworks_b200

    return opworks_b200.ops_lib()


def run(ops, logits, temps, tops, us):
    rows, vocab = logits.shape
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    ops.sample(torch.from_numpy(logits).cuda(), rows, vocab,
               torch.tensor(temps, dtype=torch.float32).cuda(), torch.tensor(tops, dtype=torch.float32).cuda(),
               torch.tensor(us, dtype=torch.float64).cuda(), out, 0)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("vocab,scale,temp,top_p", [(128256, 1.0, 0.7, 0.9), (128256, 3.0, 0.7, 0.9),
                                                    (4096, 3.0, 1.0, 1.0), (4096, 1.0, 0.7, 0.5),
                                                    (1000, 0.1, 2.0, 0.95), (50, 5.0, 0.3, 0.9)])
def test_top_p_matches_reference_rule(ops, vocab, scale, temp, top_p):
    rng = np.random.default_rng(vocab + int(100 * temp))
    rows = 32
    logits = (rng.standard_normal((rows, vocab)) * scale).astype(np.float32)
    us = rng.random(rows)
    got = run(ops, logits, [temp] * rows, [top_p] * rows, us)
    want = [oracle.top_p_sample(logits[r], temp, top_p, us[r]) for r in range(rows)]
    assert got.tolist() == want


def test_golden_sampler_cases(ops):
    g = np.load(inputs.__file__.replace("inputs.py", "sampler_golden.npz"))
    for vocab, scale, temp, top_p, seed in inputs.SAMPLER_CASES:
        logits = inputs.sampler_logits(vocab, scale, seed)
        us = np.random.default_rng(seed).random(inputs.SAMPLER_DRAWS)
        L = np.repeat(logits[None], inputs.SAMPLER_DRAWS, axis=0)
        got = run(ops, L, [temp] * len(us), [top_p] * len(us), us)
        assert got.tolist() == g[f"case{seed}"].tolist()


def test_greedy_and_edge_uniforms(ops):
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((4, 128256)).astype(np.float32)
    logits[1, [10, 20]] = 50.0  # tie for the max: lowest index wins
    got = run(ops, logits, [0.0, 0.0, 0.7, 0.7], [1.0, 1.0, 0.9, 0.9], [0.5, 0.5, 0.0, 1.0 - 2**-53])
    assert got[0] == int(np.argmax(logits[0]))
    assert got[1] == 10
    assert got[2] == oracle.top_p_sample(logits[2], 0.7, 0.9, 0.0)
    assert got[3] == oracle.top_p_sample(logits[3], 0.7, 0.9, 1.0 - 2**-53)


def test_ties_at_the_top_p_boundary(ops):
    # four equal logits straddle the cut: tokens are kept in ascending index order
    logits = np.full((1, 64), -30.0, np.float32)
    logits[0, [3, 9, 17, 40]] = 1.0
    for u in np.linspace(0, 0.999, 9):
        got = run(ops, logits, [1.0], [0.6], [u])[0]
        want = oracle.top_p_sample(logits[0], 1.0, 0.6, u)
        assert got == want
