"""Request-partitioned serving host logic (opworks_b200/serving.py) on CPU:
the LPT partition, continuous batching against a stand-in engine, and the
N-process driver as two gloo ranks (no GPU, no collective on the data path;
results gathered on rank 0)."""

import os
import socket

import numpy as np
import pytest

from opworks_b200 import serving


class FakeBatch:
    """Stand-in for LlamaBatch: token t+1 follows t; the first token encodes
    the prompt, so every request's stream is a function of the request only."""

    def __init__(self, max_batch):
        self.len = [0] * max_batch
        self.decoded_rows = []

    def reset(self, slot):
        self.len[slot] = 0

    def prefill(self, slot, ids, temperature, top_p, uniform, seed):
        assert self.len[slot] == 0, "prefill into a used slot"
        self.len[slot] = len(ids)
        return (sum(ids) + seed) % 1000

    def decode(self, slots, prev, temperature=None, top_p=None, seeds=None, steps=None):
        assert len(slots) == len(set(slots))
        for s in slots:
            assert self.len[s] > 0
            self.len[s] += 1
        self.decoded_rows.append(len(slots))
        return np.array([(p + 1) % 1000 for p in prev], np.int32)


def expected(r):
    first = (sum(r.prompt) + r.seed) % 1000
    return [(first + k) % 1000 for k in range(r.max_new_tokens)]


def test_partition_is_balanced_and_complete():
    rng = np.random.default_rng(0)
    costs = rng.integers(256 + 256, 1024 + 256, 256)
    for world in (1, 2, 4, 8):
        bins = serving.partition(costs, world)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(len(costs)))
        loads = [sum(int(costs[i]) for i in b) for b in bins]
        # LPT bound: max load <= mean + largest item
        assert max(loads) <= sum(loads) / world + max(costs)
        assert max(loads) / (sum(loads) / world) < 1.02
        assert bins == serving.partition(costs, world)  # deterministic


def test_continuous_batching_serves_every_request_once():
    reqs = [serving.Request(i, list(range(i % 7 + 3)), 1 + (i * 5) % 9, 0.7, 0.9, 100 + i) for i in range(23)]
    fb = FakeBatch(4)
    out = serving.Server(fb, 4).run(reqs)
    assert sorted(out) == list(range(23))
    for r in reqs:
        assert out[r.rid] == expected(r)
    assert max(fb.decoded_rows) <= 4
    assert sum(fb.decoded_rows) == sum(r.max_new_tokens - 1 for r in reqs)


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        reqs = serving.c5_requests(n=40, lo=8, hi=40, new_tokens=6, vocab=1000)
        res = serving.serve_partitioned(reqs, rank, world, lambda: serving.Server(FakeBatch(8), 8))
        if rank == 0:
            ok = sorted(res) == list(range(40)) and all(res[r.rid] == expected(r) for r in reqs)
            q.put(("ok" if ok else "mismatch", len(res)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(120)
def test_two_gloo_ranks_partition_and_gather():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, n = q.get(timeout=5)
    assert status == "ok" and n == 40
