"""Tensor-core (TF32 tcgen05) causal GQA prefill attention over a paged fp32
KV cache (include/ops/attention_prefill_tc.cuh, through opw_paged_attention_
prefill) against a float64 reference and against the fp32 SIMT kernel on the
same seeded inputs: ragged lengths (partial query tiles, partial pages), a
non-zero cached prefix (chunked prefill), every GQA ratio, and block tables
whose 128-key tiles are runs of consecutive blocks (staged by the 8-page run
copies) mixed with scattered pages (staged page by page). Tolerance: TF32
operands (10-bit mantissa) with fp32 accumulation, |err| <= 4e-3 (outputs are
convex combinations of V entries ~N(0,1))."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ops():
    import opworks_b200

    return opworks_b200.ops_lib()


def make_case(T, q_offset, qh, kvh, seed, extra_blocks=3, layout="scattered"):
    g = torch.Generator().manual_seed(seed)
    S = q_offset + T
    pages = (S + 15) // 16
    nblk = pages + extra_blocks
    kpool = torch.randn(nblk, kvh, 16, 64, generator=g)
    vpool = torch.randn(nblk, kvh, 16, 64, generator=g)
    perm = torch.randperm(nblk, generator=g)[:pages].int()
    if layout == "runs":  # ascending blocks from an offset: every full tile is a run
        perm = torch.arange(extra_blocks - 1, extra_blocks - 1 + pages, dtype=torch.int32)
    elif layout == "mixed":  # runs, one tile broken by a swap, a scattered tail
        perm = torch.arange(1, 1 + pages, dtype=torch.int32)
        if pages > 20:
            perm[9], perm[12] = perm[12].item(), perm[9].item()
            tail = perm[24:].clone()
            perm[24:] = tail[torch.randperm(tail.numel(), generator=g)]
    stride = pages + 1
    table = torch.full((2, stride), -1, dtype=torch.int32)
    table[1, :pages] = perm  # sequence slot 1
    q = torch.randn(T, qh * 64, generator=g)
    return q, kpool, vpool, table, stride, nblk


def reference(q, kpool, vpool, table, T, q_offset, qh, kvh):
    S = q_offset + T
    pages = (S + 15) // 16
    blk = table[1, :pages].long()
    K = kpool[blk].permute(1, 0, 2, 3).reshape(kvh, pages * 16, 64)[:, :S].double()
    V = vpool[blk].permute(1, 0, 2, 3).reshape(kvh, pages * 16, 64)[:, :S].double()
    rep = qh // kvh
    Q = q.view(T, qh, 64).permute(1, 0, 2).double()
    Kx = K.repeat_interleave(rep, dim=0)
    Vx = V.repeat_interleave(rep, dim=0)
    s = Q @ Kx.transpose(1, 2) * 0.125
    pos = torch.arange(T)[:, None] + q_offset
    mask = torch.arange(S)[None, :] > pos
    s = s.masked_fill(mask[None], float("-inf"))
    o = torch.softmax(s, dim=-1) @ Vx
    return o.permute(1, 0, 2).reshape(T, qh * 64)


def run(ops, q, kpool, vpool, table, stride, nblk, T, q_offset, qh, kvh, tc):
    out = torch.full((T, qh * 64), float("nan"), device="cuda")
    ops.paged_attention_prefill(q.cuda(), kpool.cuda(), vpool.cuda(), table.cuda(), stride, nblk, 1, T, q_offset, qh,
                                kvh, out, tc, 0)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("T,q_offset", [(1, 0), (5, 0), (33, 0), (200, 0), (129, 37), (64, 300), (1000, 0)])
def test_tc_prefill_matches_reference(ops, T, q_offset):
    qh, kvh = 32, 8
    case = make_case(T, q_offset, qh, kvh, seed=T * 7 + q_offset)
    q, kpool, vpool, table, stride, nblk = case
    want = reference(q, kpool, vpool, table, T, q_offset, qh, kvh)
    got = run(ops, *case, T, q_offset, qh, kvh, tc=1)
    assert torch.isfinite(got).all()
    err = (got.double() - want).abs().max().item()
    assert err <= 4e-3, err
    simt = run(ops, *case, T, q_offset, qh, kvh, tc=0)
    assert (simt.double() - want).abs().max().item() <= 1e-5


@pytest.mark.parametrize("qh,kvh", [(8, 8), (16, 8), (32, 8), (64, 8)])
def test_tc_prefill_gqa_ratios(ops, qh, kvh):
    T, q_offset = 77, 20
    case = make_case(T, q_offset, qh, kvh, seed=qh)
    want = reference(case[0], case[1], case[2], case[3], T, q_offset, qh, kvh)
    got = run(ops, *case, T, q_offset, qh, kvh, tc=1)
    assert torch.isfinite(got).all()
    assert (got.double() - want).abs().max().item() <= 4e-3


@pytest.mark.parametrize("layout", ["runs", "mixed"])
@pytest.mark.parametrize("T,q_offset", [(1000, 0), (129, 37), (64, 300), (300, 129), (5, 0)])
def test_tc_prefill_page_runs(ops, layout, T, q_offset):
    qh, kvh = 32, 8
    case = make_case(T, q_offset, qh, kvh, seed=T + q_offset + len(layout), layout=layout)
    want = reference(case[0], case[1], case[2], case[3], T, q_offset, qh, kvh)
    got = run(ops, *case, T, q_offset, qh, kvh, tc=1)
    assert torch.isfinite(got).all()
    assert (got.double() - want).abs().max().item() <= 4e-3
