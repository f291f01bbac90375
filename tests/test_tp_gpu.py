"""Tensor-parallel fast path on 2 GPUs (one process per GPU), with both
reductions of the o and down projections: the NCCL all-reduce, then the
fused peer-to-peer one (GEMM epilogue stores into every rank's receive
buffer over CUDA IPC mappings, rank-order sum in the residual kernel). Both
ranks return the same tokens, and they equal the single-GPU fast engine's
greedy tokens on the same prompts, with last-step logits within the
GEMM tolerance (2e-2 max-abs; the ranks' partial sums only reorder fp32
additions). Skipped on fewer than 2 GPUs."""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

STEPS = 8


def _run(b, prompts, slots):
    prev = np.array([b.prefill(i, p) for i, p in enumerate(prompts)], np.int32)
    toks = [prev]
    for _ in range(STEPS):
        prev = b.decode(slots, prev)
        toks.append(prev)
    return np.array(toks), b.logits(1)


def _worker(rank, world, id_q, handle_qs, prompts, q):
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        from opworks_b200 import pack
        from opworks_b200.llama import LlamaBatch, Model, nccl_unique_id

        # rank 0 creates the communicator id in a rank process (every rank
        # then uses the same NCCL build) and hands it to the others
        if rank == 0:
            nccl_id = nccl_unique_id()
            for _ in range(world - 1):
                id_q.put(nccl_id)
        else:
            nccl_id = id_q.get(timeout=300)

        res = {}
        with Model(pack.ensure_random_llama_pack(), weight_sets=1, device=rank) as m:
            n = len(prompts)
            slots = np.arange(n, dtype=np.int32)
            with LlamaBatch(m, n, 512, "fast", prefill_rows=256, tp=(rank, world, nccl_id)) as b:
                res["tp"], res["tp_logits"] = _run(b, prompts, slots)
                # exchange the IPC handles, switch to peer stores, run again
                mine = b.tp_ipc_handle()
                for r in range(world):
                    if r != rank:
                        handle_qs[r].put((rank, mine))
                handles = {rank: mine}
                for _ in range(world - 1):
                    r, h = handle_qs[rank].get(timeout=300)
                    handles[r] = h
                b.tp_open_peers([handles[r] for r in range(world)])
                for i in range(n):
                    b.reset(i)
                res["p2p"], res["p2p_logits"] = _run(b, prompts, slots)
            if rank == 0:
                with LlamaBatch(m, n, 512, "fast", prefill_rows=256) as b:
                    res["single"], res["single_logits"] = _run(b, prompts, slots)
        q.put((rank, res, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


def test_tensor_parallel_two_gpus_match_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from opworks_b200 import pack

    pack.ensure_random_llama_pack()  # generated once, before the ranks read it
    rng = np.random.default_rng(41)
    prompts = [rng.integers(0, 128256, int(n)).tolist() for n in (7, 64, 130, 33)]
    ctx = torch.multiprocessing.get_context("spawn")
    q, id_q = ctx.Queue(), ctx.Queue()
    handle_qs = [ctx.Queue() for _ in range(2)]
    procs = [ctx.Process(target=_worker, args=(r, 2, id_q, handle_qs, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            rank, res, err = q.get(timeout=600)
            assert err is None, f"rank {rank}: {err}"
            out[rank] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for path in ("tp", "p2p"):
        assert np.array_equal(out[0][path], out[1][path]), path
        assert np.array_equal(out[0][path], out[0]["single"]), (path, out[0][path], out[0]["single"])
        err = np.max(np.abs(out[0][path + "_logits"] - out[0]["single_logits"]))
        assert err <= 2e-2, (path, err)
    # both reductions add the same two partial sums: identical logits
    assert np.array_equal(out[0]["p2p_logits"], out[1]["p2p_logits"])
