"""Request-partitioned serving (benchmark config C5): requests are independent, so N
GPUs serve disjoint subsets of them, one process per GPU, with no collective
on the data path. Each process runs continuous batching over one LlamaBatch
(paged KV cache, CUDA-graph decode steps, device sampling); results are
gathered on rank 0 over torch.distributed (gloo or NCCL) after the work.

    partition(costs, world)            deterministic LPT assignment
    Request / Server.run(requests)     continuous batching on one GPU
    serve_partitioned(requests, ...)   the N-process driver
"""

from __future__ import annotations

import dataclasses
import heapq
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np


@dataclasses.dataclass
class Request:
    rid: int
    prompt: Sequence[int]
    max_new_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    seed: int = 0

    @property
    def cost(self) -> int:
        # work of a request ~ tokens it moves through the model
        return len(self.prompt) + self.max_new_tokens


def partition(costs: Sequence[int], world: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of items to `world` bins:
    items in decreasing cost (ties by index) each go to the least loaded bin
    (ties by bin index). Deterministic, so every rank computes the same split
    without communicating. Returns each bin's item indices in increasing order."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    heap = [(0, b) for b in range(world)]
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, b = heapq.heappop(heap)
        bins[b].append(i)
        heapq.heappush(heap, (load + int(costs[i]), b))
    return [sorted(x) for x in bins]


class Server:
    """Continuous batching on one GPU: up to `max_batch` requests hold a KV slot
    each; every step admits pending requests into free slots (prefill returns
    their first token), then decodes all active slots together and retires the
    requests that reached max_new_tokens (or an EOS id when stop_at_eos)."""

    def __init__(self, batch, max_batch: int, eos: Optional[Sequence[int]] = None, stop_at_eos: bool = False):
        self.batch = batch  # opworks_b200.llama.LlamaBatch (or a stand-in with the same methods)
        self.max_batch = max_batch
        self.eos = set(int(x) for x in (eos or ()))
        self.stop_at_eos = stop_at_eos
        self.steps = 0
        self.prefill_tokens = 0
        self.decode_tokens = 0

    def run(self, requests: Sequence[Request]) -> Dict[int, List[int]]:
        pending = list(requests)[::-1]
        free = list(range(self.max_batch))[::-1]
        active: Dict[int, Request] = {}  # slot -> request
        out: Dict[int, List[int]] = {}
        last: Dict[int, int] = {}
        while pending or active:
            while pending and free:
                r = pending.pop()
                slot = free.pop()
                self.batch.reset(slot)
                tok = self.batch.prefill(slot, list(r.prompt), r.temperature, r.top_p, -1.0, r.seed)
                self.prefill_tokens += len(r.prompt)
                out[r.rid] = [int(tok)]
                if self._done(r, out[r.rid]):
                    free.append(slot)
                    continue
                active[slot] = r
                last[slot] = int(tok)
            if not active:
                continue
            slots = sorted(active)
            reqs = [active[s] for s in slots]
            toks = self.batch.decode(slots, [last[s] for s in slots],
                                     temperature=np.array([r.temperature for r in reqs], np.float32),
                                     top_p=np.array([r.top_p for r in reqs], np.float32),
                                     seeds=np.array([r.seed for r in reqs], np.uint64),
                                     steps=np.array([len(out[r.rid]) for r in reqs], np.int32))
            self.steps += 1
            self.decode_tokens += len(slots)
            for s, r, t in zip(slots, reqs, toks):
                out[r.rid].append(int(t))
                last[s] = int(t)
                if self._done(r, out[r.rid]):
                    del active[s]
                    free.append(s)
        return out

    def _done(self, r: Request, toks: List[int]) -> bool:
        return len(toks) >= r.max_new_tokens or (self.stop_at_eos and toks[-1] in self.eos)


def serve_partitioned(requests: Sequence[Request], rank: int, world: int,
                      make_server: Callable[[], Server], gather: bool = True) -> Optional[Dict[int, List[int]]]:
    """Serve this rank's share of `requests`; with `gather`, rank 0 returns the
    tokens of every request (torch.distributed.gather_object), others None."""
    shares = partition([r.cost for r in requests], world)
    mine = [requests[i] for i in shares[rank]]
    result = make_server().run(mine) if mine else {}
    if world == 1 or not gather:
        return result
    import torch.distributed as dist

    parts = [None] * world if rank == 0 else None
    dist.gather_object(result, parts, dst=0)
    if rank != 0:
        return None
    merged: Dict[int, List[int]] = {}
    for p in parts:
        merged.update(p)
    return merged


def c5_requests(n=256, lo=256, hi=1024, new_tokens=256, vocab=128256, temperature=0.7, top_p=0.9, seed=9):
    """Config C5: `n` requests, prompt lengths uniform in [lo, hi], uniform
    random ids, `new_tokens` sampled tokens each."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, n)
    return [Request(i, rng.integers(0, vocab, int(L)).astype(np.int32).tolist(), new_tokens, temperature, top_p,
                    seed * 100_000 + i) for i, L in enumerate(lens)]
