"""Host-sync-free multi-step decode (opw_llama_batch_decode_multi): `steps`
graph replays with the sampled tokens fed back on the device give exactly the
tokens of `steps` single-step calls with the same sampling arguments (counter
RNG and explicit uniforms, greedy and top-p), the KV cache ends in the same
state (the next single step agrees), and a row stops counting at its eos."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")

N, STEPS = 4, 12


@pytest.fixture(scope="module")
def model():
    from opworks_b200 import pack
    from opworks_b200.llama import Model

    with Model(pack.ensure_random_llama_pack(), weight_sets=1) as m:
        yield m


def prefill_all(b, prompts, temp, seeds):
    return np.array([b.prefill(i, p, temp, 0.9, -1.0, int(seeds[i])) for i, p in enumerate(prompts)], np.int32)


@pytest.mark.parametrize("temp,explicit", [(0.0, False), (0.7, False), (0.7, True)])
def test_multi_step_equals_single_steps(model, temp, explicit):
    from opworks_b200.llama import LlamaBatch

    rng = np.random.default_rng(31)
    prompts = [rng.integers(0, model.vocab, int(n)).tolist() for n in (5, 17, 40, 33)]
    seeds = (900 + np.arange(N)).astype(np.uint64)
    uni = rng.random((STEPS + 1, N)) if explicit else None
    slots = np.arange(N, dtype=np.int32)
    with LlamaBatch(model, N, 256, "fast", prefill_rows=64) as b:
        prev = prefill_all(b, prompts, temp, seeds)
        single = []
        t = prev
        for k in range(STEPS):
            t = b.decode(slots, t, temperature=temp, top_p=0.9, seeds=seeds, steps=k + 1,
                         uniforms=uni[k] if explicit else None)
            single.append(t)
        single = np.array(single)
        nxt_single = b.decode(slots, t, temperature=temp, top_p=0.9, seeds=seeds, steps=STEPS + 1,
                              uniforms=uni[STEPS] if explicit else None)
        for i in range(N):
            b.reset(i)
        prev2 = prefill_all(b, prompts, temp, seeds)
        assert np.array_equal(prev, prev2)
        multi, counts = b.decode_multi(slots, prev2, STEPS, temperature=temp, top_p=0.9, seeds=seeds,
                                       steps0=1, uniforms=uni[:STEPS] if explicit else None)
        assert np.array_equal(multi, single), (multi, single)
        assert np.all(counts == STEPS)
        # the KV cache and lengths advanced exactly as with single steps
        nxt_multi = b.decode(slots, multi[-1], temperature=temp, top_p=0.9, seeds=seeds, steps=STEPS + 1,
                             uniforms=uni[STEPS] if explicit else None)
        assert np.array_equal(nxt_multi, nxt_single)


def test_multi_step_eos_stops_count(model):
    from opworks_b200.llama import LlamaBatch

    rng = np.random.default_rng(32)
    prompts = [rng.integers(0, model.vocab, 24).tolist() for _ in range(N)]
    seeds = (700 + np.arange(N)).astype(np.uint64)
    slots = np.arange(N, dtype=np.int32)
    with LlamaBatch(model, N, 256, "fast", prefill_rows=64) as b:
        prev = prefill_all(b, prompts, 0.7, seeds)
        ref, _ = b.decode_multi(slots, prev, STEPS, temperature=0.7, top_p=0.9, seeds=seeds, steps0=1)
        for i in range(N):
            b.reset(i)
        prev = prefill_all(b, prompts, 0.7, seeds)
        eos = int(ref[5, 1])  # row 1 emits it at step 5 (maybe earlier, maybe in other rows)
        got, counts = b.decode_multi(slots, prev, STEPS, temperature=0.7, top_p=0.9, seeds=seeds, steps0=1,
                                     eos_id=eos)
        for i in range(N):
            hits = np.nonzero(ref[:, i] == eos)[0]
            stop = int(hits[0]) + 1 if hits.size else STEPS
            assert counts[i] == stop
            assert np.array_equal(got[:stop, i], ref[:stop, i])
            assert np.all(got[stop:, i] == -1)


def test_multi_step_call_lengths_share_and_regrow_graphs(model):
    """Calls of 4, 300 and again 4 steps (explicit uniforms): the 300-step
    call outgrows the token and uniform buffers (257 step rows), which
    recaptures the multi-step graph; every call still gives the tokens of
    single-step calls with the same uniforms."""
    from opworks_b200.llama import LlamaBatch

    n = 2
    lengths = (4, 300, 4)
    total = sum(lengths)
    rng = np.random.default_rng(33)
    prompts = [rng.integers(0, model.vocab, 20).tolist() for _ in range(n)]
    uni = rng.random((total, n))
    seeds = (900 + np.arange(n)).astype(np.uint64)
    slots = np.arange(n, dtype=np.int32)
    with LlamaBatch(model, n, 20 + total + 8, "fast", prefill_rows=32) as b:
        prev = prefill_all(b, prompts, 0.7, seeds)
        multi, k = [], 0
        for length in lengths:
            toks, counts = b.decode_multi(slots, prev, length, temperature=0.7, top_p=0.9, uniforms=uni[k:k + length],
                                          seeds=seeds, steps0=1 + k)
            assert np.all(counts == length)
            multi.append(toks)
            prev = toks[-1]
            k += length
        multi = np.concatenate(multi)
    with LlamaBatch(model, n, 20 + total + 8, "fast", prefill_rows=32) as b:
        t = prefill_all(b, prompts, 0.7, seeds)
        single = []
        for k in range(total):
            t = b.decode(slots, t, temperature=0.7, top_p=0.9, uniforms=uni[k], seeds=seeds, steps=k + 1)
            single.append(t)
    assert np.array_equal(multi, np.array(single))
